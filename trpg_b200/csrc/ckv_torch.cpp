// torch.library registration of the compressed-KV ops (namespace `ckv`).
//
// A thin layer: it checks tensor shapes, dtypes and devices, reads strides,
// picks the current CUDA stream and calls the C ABI of libtrpg_ckv.so.  No
// computation happens here and there is no CPU implementation.
#include <ATen/ATen.h>
#include <ATen/autocast_mode.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <atomic>
#include <map>
#include <mutex>
#include <tuple>
#include <utility>
#include <vector>

#include "ckv.h"

namespace {

using at::Tensor;

void check_status(int st, const char *what) {
  TORCH_CHECK(st == CKV_OK, "ckv::", what, " failed: ", ckv_status_string(st),
              (st == CKV_ERR_CUDA ? std::string(" (") + ckv_last_error() + ")" : std::string()));
}

int dtype_code(at::ScalarType t) {
  if (t == at::kBFloat16) return CKV_BF16;
  if (t == at::kHalf) return CKV_F16;
  TORCH_CHECK(false, "ckv: expected bfloat16 or float16, got ", t);
  return -1;
}

ckv_stream_t current_stream(const Tensor &t) {
  return reinterpret_cast<ckv_stream_t>(c10::cuda::getCurrentCUDAStream(t.get_device()).stream());
}

void require_cuda(const Tensor &t, const char *name) {
  TORCH_CHECK(t.is_cuda(), "ckv: ", name, " must be a CUDA tensor (this library has no CPU path)");
}

// ---------------------------------------------------------------------------
// Quantizer
// ---------------------------------------------------------------------------
std::tuple<Tensor, Tensor> pack_rows(const Tensor &rows, int64_t bits, int64_t rounding) {
  require_cuda(rows, "rows");
  TORCH_CHECK(rows.dim() >= 1, "ckv::pack_rows: rows must have a group dimension");
  const int64_t group = rows.size(-1);
  TORCH_CHECK(group == 64 || group == 128, "ckv::pack_rows: group must be 64 or 128, got ", group);
  TORCH_CHECK(bits == 4 || bits == 8, "ckv::pack_rows: bits must be 4 or 8");
  c10::cuda::CUDAGuard guard(rows.device());
  Tensor x = rows.contiguous();
  auto shape = x.sizes().vec();
  shape.back() = group * bits / 8;
  Tensor codes = at::empty(shape, x.options().dtype(at::kByte));
  shape.back() = 2;
  Tensor meta = at::empty(shape, x.options().dtype(at::kFloat));
  const int64_t n = x.numel() / group;
  check_status(ckv_pack_rows(x.data_ptr(), dtype_code(x.scalar_type()), n, int(group), int(bits),
                             int(rounding), codes.data_ptr<uint8_t>(), meta.data_ptr<float>(),
                             current_stream(x)),
               "pack_rows");
  return {codes, meta};
}

Tensor unpack_rows(const Tensor &data, const Tensor &meta, int64_t bits, at::ScalarType dtype) {
  require_cuda(data, "data");
  require_cuda(meta, "meta");
  TORCH_CHECK(data.scalar_type() == at::kByte && meta.scalar_type() == at::kFloat,
              "ckv::unpack_rows: data must be uint8 and meta float32");
  TORCH_CHECK(bits == 4 || bits == 8, "ckv::unpack_rows: bits must be 4 or 8");
  c10::cuda::CUDAGuard guard(data.device());
  Tensor d = data.contiguous(), m = meta.contiguous();
  const int64_t group = d.size(-1) * (bits == 4 ? 2 : 1);
  TORCH_CHECK(m.size(-1) == 2 && m.numel() * group / 2 == d.numel() * (bits == 4 ? 2 : 1),
              "ckv::unpack_rows: meta must hold (scale, low) per row");
  auto shape = d.sizes().vec();
  shape.back() = group;
  Tensor out = at::empty(shape, d.options().dtype(dtype));
  check_status(ckv_unpack_rows(d.data_ptr<uint8_t>(), m.data_ptr<float>(), d.numel() * 8 / bits / group,
                               int(group), int(bits), dtype_code(dtype), out.data_ptr(),
                               current_stream(d)),
               "unpack_rows");
  return out;
}

// Quantize residual tokens [0, count) of keys/values [1,H,R,D] into the banks
// at unit `unit_offset`.  Banks: key [1,H,U,D,S], value [1,H,T,D/64,S'].
void pack_append(const Tensor &keys, const Tensor &values, const Tensor &kd, const Tensor &km,
                 const Tensor &vd, const Tensor &vm, int64_t count, int64_t unit_offset,
                 int64_t bits, int64_t rounding) {
  for (auto *t : {&keys, &values, &kd, &km, &vd, &vm}) require_cuda(*t, "append tensor");
  TORCH_CHECK(keys.dim() == 4 && values.sizes() == keys.sizes() && keys.size(0) == 1,
              "ckv::pack_append: keys/values must be [1,H,R,D]");
  TORCH_CHECK(keys.scalar_type() == values.scalar_type(), "ckv::pack_append: dtype mismatch");
  TORCH_CHECK(keys.stride(-1) == 1 && values.stride(-1) == 1, "ckv::pack_append: last dim dense");
  TORCH_CHECK(count >= 0 && count % 128 == 0 && count <= keys.size(2),
              "ckv::pack_append: count must be a multiple of 128 within the residual");
  const int64_t H = keys.size(1), D = keys.size(3), S = 128 * bits / 8, SV = 64 * bits / 8;
  TORCH_CHECK(kd.dim() == 5 && kd.size(1) == H && kd.size(3) == D && kd.size(4) == S &&
                  kd.stride(4) == 1 && kd.stride(3) == S && kd.scalar_type() == at::kByte,
              "ckv::pack_append: key bank must be uint8 [1,H,U,D,", S, "] with dense inner dims");
  TORCH_CHECK(km.dim() == 5 && km.size(1) == H && km.size(3) == D && km.size(4) == 2 &&
                  km.stride(4) == 1 && km.stride(3) == 2 && km.scalar_type() == at::kFloat,
              "ckv::pack_append: key meta must be float32 [1,H,U,D,2]");
  TORCH_CHECK(vd.dim() == 5 && vd.size(1) == H && vd.size(3) == D / 64 && vd.size(4) == SV &&
                  vd.stride(4) == 1 && vd.stride(3) == SV && vd.scalar_type() == at::kByte,
              "ckv::pack_append: value bank must be uint8 [1,H,T,D/64,", SV, "]");
  TORCH_CHECK(vm.dim() == 5 && vm.size(1) == H && vm.size(3) == D / 64 && vm.size(4) == 2 &&
                  vm.stride(4) == 1 && vm.stride(3) == 2 && vm.scalar_type() == at::kFloat,
              "ckv::pack_append: value meta must be float32 [1,H,T,D/64,2]");
  TORCH_CHECK(unit_offset >= 0 && unit_offset + count / 128 <= kd.size(2) &&
                  unit_offset + count / 128 <= km.size(2) &&
                  (unit_offset * 128 + count) <= vd.size(2) && (unit_offset * 128 + count) <= vm.size(2),
              "ckv::pack_append: bank capacity exceeded");
  if (count == 0) return;
  c10::cuda::CUDAGuard guard(keys.device());
  ckv_append_args a{};
  a.keys = keys.data_ptr();
  a.values = values.data_ptr();
  a.k_stride_head = keys.stride(1);
  a.k_stride_token = keys.stride(2);
  a.v_stride_head = values.stride(1);
  a.v_stride_token = values.stride(2);
  a.key_data = kd.data_ptr<uint8_t>();
  a.key_meta = km.data_ptr<float>();
  a.value_data = vd.data_ptr<uint8_t>();
  a.value_meta = vm.data_ptr<float>();
  a.kd_stride_head = kd.stride(1);
  a.kd_stride_unit = kd.stride(2);
  a.km_stride_head = km.stride(1);
  a.km_stride_unit = km.stride(2);
  a.vd_stride_head = vd.stride(1);
  a.vd_stride_token = vd.stride(2);
  a.vm_stride_head = vm.stride(1);
  a.vm_stride_token = vm.stride(2);
  a.heads = int(H);
  a.head_dim = int(D);
  a.bits = int(bits);
  a.dtype = dtype_code(keys.scalar_type());
  a.rounding = int(rounding);
  a.count = int(count);
  a.unit_offset = int(unit_offset);
  check_status(ckv_pack_append(&a, current_stream(keys)), "pack_append");
}

// Layouts the kernels need.  A tensor that already has it passes through; any
// other (a strided view, a misaligned base) is copied once here.
bool aligned16(const Tensor &t) { return (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0; }

Tensor fit_copy(const Tensor &t) {
  Tensor c = t.contiguous();
  return aligned16(c) ? c : c.clone();
}

// Bank tensor: the last `dense` dims packed densely, 16-byte aligned base.
Tensor fit_bank(const Tensor &t, int dense) {
  if (!t.defined()) return t;
  const int64_t d = t.dim();
  bool ok = d >= dense && t.stride(d - 1) == 1 && aligned16(t);
  int64_t expect = t.size(d - 1);
  for (int k = 2; ok && k <= dense; ++k) {
    ok = t.stride(d - k) == expect;
    expect *= t.size(d - k);
  }
  return ok ? t : fit_copy(t);
}

// Rows of 16-bit values: last dim dense, head and token strides multiples of
// 8 elements (16-byte rows), 16-byte aligned base.
Tensor fit_rows(const Tensor &t) {
  if (!t.defined() || t.dim() != 4) return t;
  const bool ok = t.stride(3) == 1 && t.stride(1) % 8 == 0 && t.stride(2) % 8 == 0 && aligned16(t);
  return ok ? t : fit_copy(t);
}

// A window view [1,H,r,D] whose rows sit in a buffer of `capacity` rows per
// head: dense rows of D elements, heads `capacity * D` apart, and a storage
// large enough for all of them.  Anything else is not a window this op may
// write past the end of.
bool window_holds(const Tensor &w, int64_t capacity) {
  if (w.dim() != 4 || w.size(0) != 1 || w.stride(3) != 1 || w.stride(2) != w.size(3)) return false;
  const int64_t H = w.size(1), D = w.size(3);
  if (H > 1 && w.stride(1) != capacity * D) return false;
  const int64_t need = w.storage_offset() + (H - 1) * capacity * D + capacity * D;
  return int64_t(w.storage().nbytes()) >= need * int64_t(w.element_size());
}

// keys[:, :, offset:offset+n] = keys_new (and values) for window buffers
// [1,H,C,D] with capacity C >= offset + n; one launch.
// Writes the new rows at `offset` and returns the window views of the rows
// written so far (the first offset + n rows of each buffer).
std::tuple<Tensor, Tensor> residual_append(const Tensor &keys_new, const Tensor &values_new,
                                           const Tensor &keys, const Tensor &values, int64_t offset) {
  for (auto *t : {&keys_new, &values_new, &keys, &values}) require_cuda(*t, "residual tensor");
  TORCH_CHECK(keys_new.dim() == 4 && values_new.sizes() == keys_new.sizes() && keys_new.size(0) == 1,
              "ckv::residual_append: new rows must be [1,H,n,D]");
  TORCH_CHECK(keys.dim() == 4 && values.sizes() == keys.sizes() && keys.size(0) == 1 &&
                  keys.size(1) == keys_new.size(1) && keys.size(3) == keys_new.size(3),
              "ckv::residual_append: window buffers must be [1,H,C,D]");
  for (auto *t : {&values_new, &keys, &values}) {
    TORCH_CHECK(t->scalar_type() == keys_new.scalar_type(), "ckv::residual_append: dtype mismatch");
    TORCH_CHECK(t->device() == keys_new.device(), "ckv::residual_append: device mismatch");
  }
  TORCH_CHECK(offset >= 0 && offset + keys_new.size(2) <= keys.size(2),
              "ckv::residual_append: window capacity exceeded");
  c10::cuda::CUDAGuard guard(keys.device());
  const Tensor kn = fit_rows(keys_new), vn = fit_rows(values_new);
  ckv_residual_args a{};
  a.keys_new = kn.data_ptr();
  a.values_new = vn.data_ptr();
  a.kn_stride_head = kn.stride(1);
  a.kn_stride_token = kn.stride(2);
  a.vn_stride_head = vn.stride(1);
  a.vn_stride_token = vn.stride(2);
  a.keys = keys.data_ptr();
  a.values = values.data_ptr();
  a.k_stride_head = keys.stride(1);
  a.k_stride_token = keys.stride(2);
  a.v_stride_head = values.stride(1);
  a.v_stride_token = values.stride(2);
  a.heads = int(keys.size(1));
  a.tokens = int(keys_new.size(2));
  a.head_dim = int(keys.size(3));
  a.offset = int(offset);
  TORCH_CHECK(keys.stride(3) == 1 && values.stride(3) == 1 && aligned16(keys) && aligned16(values) &&
                  keys.stride(1) % 8 == 0 && keys.stride(2) % 8 == 0 && values.stride(1) % 8 == 0 &&
                  values.stride(2) % 8 == 0,
              "ckv::residual_append: window buffers need dense, 16-byte aligned rows");
  check_status(ckv_residual_append(&a, current_stream(keys)), "residual_append");
  const int64_t rows = offset + keys_new.size(2);
  return {keys.narrow(2, 0, rows), values.narrow(2, 0, rows)};
}

// Append to the exact window in place: `keys` / `values` are the current
// window views [1,H,r,D] of buffers with `capacity` rows per head.  The new
// rows go to rows [r, r + n) (past the end of the views, so views handed out
// earlier keep their contents) and the views of the first r + n rows come
// back.  The buffer geometry is re-derived from the views and checked against
// their storage before anything is written.
std::tuple<Tensor, Tensor> window_append(const Tensor &keys_new, const Tensor &values_new,
                                         const Tensor &keys, const Tensor &values,
                                         int64_t capacity) {
  TORCH_CHECK(keys.dim() == 4 && values.sizes() == keys.sizes(),
              "ckv::window_append: window views must be [1,H,r,D]");
  TORCH_CHECK(window_holds(keys, capacity) && window_holds(values, capacity),
              "ckv::window_append: the views are not rows of a window buffer of capacity ", capacity);
  const int64_t H = keys.size(1), D = keys.size(3), r = keys.size(2);
  const std::vector<int64_t> full{1, H, capacity, D}, st{H * capacity * D, capacity * D, D, 1};
  const Tensor kb = keys.as_strided(full, st, keys.storage_offset());
  const Tensor vb = values.as_strided(full, st, values.storage_offset());
  return residual_append(keys_new, values_new, kb, vb, r);
}

// ---------------------------------------------------------------------------
// Attention
// ---------------------------------------------------------------------------

// One persistent workspace per (device, stream): calls on one stream are
// ordered, and every call leaves the counter region at zero.
struct Workspace {
  std::mutex mu;
  std::map<std::pair<int, cudaStream_t>, Tensor> buffers;
};
Workspace &workspaces() {
  static Workspace *w = new Workspace();
  return *w;
}

Tensor workspace_for(const Tensor &like, size_t bytes) {
  auto stream = c10::cuda::getCurrentCUDAStream(like.get_device());
  auto key = std::make_pair(int(like.get_device()), stream.stream());
  auto &ws = workspaces();
  std::lock_guard<std::mutex> lock(ws.mu);
  auto it = ws.buffers.find(key);
  if (it != ws.buffers.end() && size_t(it->second.numel()) >= bytes) return it->second;
  cudaStreamCaptureStatus status = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(stream.stream(), &status);
  TORCH_CHECK(status == cudaStreamCaptureStatusNone,
              "ckv: the attention workspace must be allocated before stream capture; run one "
              "call of the same (or larger) size on this stream first");
  size_t cap = std::max<size_t>(bytes, size_t(1) << 20);
  cap = (cap + (1 << 20) - 1) / (1 << 20) * (1 << 20);
  Tensor t = at::zeros({int64_t(cap)}, like.options().dtype(at::kByte));
  ws.buffers[key] = t;
  return t;
}

ckv_seq make_seq(const Tensor &q, const Tensor &kd, const Tensor &km, const Tensor &vd,
                 const Tensor &vm, const Tensor &rk, const Tensor &rv, int64_t packed,
                 int64_t length, const int64_t *range, int64_t bits, int64_t hkv) {
  const int64_t D = q.size(3), S = 128 * bits / 8, SV = 64 * bits / 8;
  ckv_seq s{};
  s.query = q.data_ptr();
  s.q_stride_head = q.stride(1);
  s.q_stride_pos = q.stride(2);
  s.packed_tokens = packed;
  s.length = length;
  s.unit_begin = int32_t(range[0]);
  s.unit_end = int32_t(range[1]);
  s.resid_begin = int32_t(range[2]);
  s.resid_end = int32_t(range[3]);
  if (range[1] > range[0]) {
    TORCH_CHECK(kd.defined() && km.defined() && vd.defined() && vm.defined(),
                "ckv::attention: packed range needs the banks");
    TORCH_CHECK(kd.scalar_type() == at::kByte && vd.scalar_type() == at::kByte &&
                    km.scalar_type() == at::kFloat && vm.scalar_type() == at::kFloat,
                "ckv::attention: banks must be uint8 codes with float32 meta");
    TORCH_CHECK(kd.dim() == 5 && kd.size(1) == hkv && kd.size(3) == D && kd.size(4) == S &&
                    kd.stride(4) == 1 && kd.stride(3) == S && kd.size(2) >= range[1],
                "ckv::attention: key codes must be [1,H,U,D,", S, "] with dense inner dims");
    TORCH_CHECK(km.dim() == 5 && km.size(1) == hkv && km.size(3) == D && km.size(4) == 2 &&
                    km.stride(4) == 1 && km.stride(3) == 2 && km.size(2) >= range[1],
                "ckv::attention: key meta must be [1,H,U,D,2] with dense inner dims");
    TORCH_CHECK(vd.dim() == 5 && vd.size(1) == hkv && vd.size(3) == D / 64 && vd.size(4) == SV &&
                    vd.stride(4) == 1 && vd.stride(3) == SV && vd.size(2) >= range[1] * 128,
                "ckv::attention: value codes must be [1,H,T,D/64,", SV, "] with dense inner dims");
    TORCH_CHECK(vm.dim() == 5 && vm.size(1) == hkv && vm.size(3) == D / 64 && vm.size(4) == 2 &&
                    vm.stride(4) == 1 && vm.stride(3) == 2 && vm.size(2) >= range[1] * 128,
                "ckv::attention: value meta must be [1,H,T,D/64,2] with dense inner dims");
    s.key_data = kd.data_ptr<uint8_t>();
    s.kd_stride_head = kd.stride(1);
    s.kd_stride_unit = kd.stride(2);
    s.key_meta = km.data_ptr<float>();
    s.km_stride_head = km.stride(1);
    s.km_stride_unit = km.stride(2);
    s.value_data = vd.data_ptr<uint8_t>();
    s.vd_stride_head = vd.stride(1);
    s.vd_stride_token = vd.stride(2);
    s.value_meta = vm.data_ptr<float>();
    s.vm_stride_head = vm.stride(1);
    s.vm_stride_token = vm.stride(2);
  }
  if (range[3] > range[2]) {
    TORCH_CHECK(rk.defined() && rv.defined() && rk.dim() == 4 && rv.sizes() == rk.sizes() &&
                    rk.size(1) == hkv && rk.size(3) == D && rk.size(2) >= range[3] &&
                    rk.stride(3) == 1 && rv.stride(3) == 1 &&
                    rk.scalar_type() == q.scalar_type() && rv.scalar_type() == q.scalar_type(),
                "ckv::attention: residual must be [1,H,R,D] in the query dtype, last dim dense");
    s.keys = rk.data_ptr();
    s.rk_stride_head = rk.stride(1);
    s.rk_stride_token = rk.stride(2);
    s.values = rv.data_ptr();
    s.rv_stride_head = rv.stride(1);
    s.rv_stride_token = rv.stride(2);
  }
  return s;
}

void run_attention(std::vector<ckv_seq> &seqs, const Tensor &q0, int64_t hq, int64_t hkv, int64_t D,
                   int64_t nq, int64_t bits, double scale, bool partial);

// Dequantization rule of the attention ops in this process: 0 exact (the
// reference's per-element rounding), 1 folded (CKV_DEQUANT_FOLDED).
std::atomic<int> g_dequant{0};

int64_t set_dequant(int64_t mode) {
  TORCH_CHECK(mode == 0 || mode == 1, "ckv::set_dequant: mode must be 0 (exact) or 1 (folded)");
  return g_dequant.exchange(int(mode));
}

// queries[i]: [1,Hq,nq,D]; banks and residuals per sequence; ranges[i*4..] =
// (unit_begin, unit_end, resid_begin, resid_end).  Returns one tensor per
// sequence: [1,Hq,nq,D] in the query dtype, or [Hq*nq, D+2] fp32 partials.
std::vector<Tensor> attention(const std::vector<Tensor> &queries, const std::vector<Tensor> &kd,
                              const std::vector<Tensor> &km, const std::vector<Tensor> &vd,
                              const std::vector<Tensor> &vm, const std::vector<Tensor> &rk,
                              const std::vector<Tensor> &rv, std::vector<int64_t> packed,
                              std::vector<int64_t> lengths, std::vector<int64_t> ranges,
                              int64_t bits, double scale, bool partial) {
  const size_t n = queries.size();
  TORCH_CHECK(n >= 1 && n <= CKV_MAX_SEQS, "ckv::attention: 1..", CKV_MAX_SEQS, " sequences per call");
  TORCH_CHECK(kd.size() == n && km.size() == n && vd.size() == n && vm.size() == n &&
                  rk.size() == n && rv.size() == n && packed.size() == n && lengths.size() == n &&
                  ranges.size() == 4 * n,
              "ckv::attention: per-sequence argument lists must have equal length");
  const Tensor &q0 = queries[0];
  require_cuda(q0, "query");
  TORCH_CHECK(q0.dim() == 4 && q0.size(0) == 1 && q0.stride(3) == 1,
              "ckv::attention: query must be [1,Hq,nq,D] with a dense last dim");
  const int64_t hq = q0.size(1), nq = q0.size(2), D = q0.size(3);
  int64_t hkv = 0;
  for (size_t i = 0; i < n; ++i) {
    if (ranges[4 * i + 1] > ranges[4 * i]) { hkv = kd[i].size(1); break; }
    if (ranges[4 * i + 3] > ranges[4 * i + 2]) { hkv = rk[i].size(1); break; }
  }
  TORCH_CHECK(hkv > 0, "ckv::attention: every sequence range is empty");
  c10::cuda::CUDAGuard guard(q0.device());
  std::vector<ckv_seq> seqs(n);
  std::vector<Tensor> outs(n);
  std::vector<Tensor> keep;   // layout copies made for this call
  keep.reserve(6 * n);
  for (size_t i = 0; i < n; ++i) {
    const Tensor &q = queries[i];
    TORCH_CHECK(q.device() == q0.device() && q.scalar_type() == q0.scalar_type() &&
                    q.sizes() == q0.sizes() && q.stride(3) == 1,
                "ckv::attention: queries must share device, dtype and shape");
    for (const Tensor *t : {&kd[i], &km[i], &vd[i], &vm[i], &rk[i], &rv[i]})
      TORCH_CHECK(!t->defined() || t->device() == q0.device(),
                  "ckv::attention: all tensors must be on the query's device");
    const bool has_packed = ranges[4 * i + 1] > ranges[4 * i];
    const bool has_resid = ranges[4 * i + 3] > ranges[4 * i + 2];
    keep.push_back(has_packed ? fit_bank(kd[i], 2) : Tensor());
    keep.push_back(has_packed ? fit_bank(km[i], 2) : Tensor());
    keep.push_back(has_packed ? fit_bank(vd[i], 3) : Tensor());
    keep.push_back(has_packed ? fit_bank(vm[i], 3) : Tensor());
    keep.push_back(has_resid ? fit_rows(rk[i]) : Tensor());
    keep.push_back(has_resid ? fit_rows(rv[i]) : Tensor());
    const Tensor *f = &keep[keep.size() - 6];
    seqs[i] = make_seq(q, f[0], f[1], f[2], f[3], f[4], f[5], packed[i], lengths[i],
                       &ranges[4 * i], bits, hkv);
    outs[i] = partial ? at::empty({hq * nq, D + 2}, q.options().dtype(at::kFloat))
                      : at::empty({1, hq, nq, D}, q.options());
    seqs[i].out = outs[i].data_ptr();
  }
  run_attention(seqs, q0, hq, hkv, D, nq, bits, scale, partial);
  return outs;
}

void run_attention(std::vector<ckv_seq> &seqs, const Tensor &q0, int64_t hq, int64_t hkv, int64_t D,
                   int64_t nq, int64_t bits, double scale, bool partial) {
  const size_t n = seqs.size();
  ckv_attn_args a{};
  a.seqs = seqs.data();
  a.num_seqs = int32_t(n);
  a.heads_q = int32_t(hq);
  a.heads_kv = int32_t(hkv);
  a.head_dim = int32_t(D);
  a.nq = int32_t(nq);
  a.bits = int32_t(bits);
  a.dtype = dtype_code(q0.scalar_type());
  a.scale = float(scale);
  a.partial = partial ? 1 : 0;
  a.flags = CKV_WS_COUNTERS_ZERO | (g_dequant.load(std::memory_order_relaxed) ? CKV_DEQUANT_FOLDED : 0);
  size_t bytes = 0;
  check_status(ckv_attention_workspace(&a, &bytes), "attention_workspace");
  Tensor ws = workspace_for(q0, bytes);
  check_status(ckv_attention(&a, ws.data_ptr(), size_t(ws.numel()), current_stream(q0)), "attention");
}

// Single sequence, plain tensors: the decode / verify fast path.
Tensor decode(const Tensor &q, const Tensor &kd, const Tensor &km, const Tensor &vd,
              const Tensor &vm, const Tensor &rk, const Tensor &rv, int64_t packed, int64_t length,
              int64_t bits, double scale) {
  require_cuda(q, "query");
  TORCH_CHECK(q.dim() == 4 && q.size(0) == 1 && q.stride(3) == 1,
              "ckv::decode: query must be [1,Hq,nq,D] with a dense last dim");
  for (const Tensor *t : {&kd, &km, &vd, &vm, &rk, &rv})
    TORCH_CHECK(t->device() == q.device(), "ckv::decode: all tensors must be on the query's device");
  c10::cuda::CUDAGuard guard(q.device());
  const int64_t range[4] = {0, packed / 128, 0, rk.size(2)};
  const int64_t hkv = rk.size(1);
  const Tensor kd2 = fit_bank(kd, 2), km2 = fit_bank(km, 2), vd2 = fit_bank(vd, 3),
               vm2 = fit_bank(vm, 3), rk2 = fit_rows(rk), rv2 = fit_rows(rv);
  std::vector<ckv_seq> seqs(1);
  seqs[0] = make_seq(q, kd2, km2, vd2, vm2, rk2, rv2, packed, length, range, bits, hkv);
  Tensor out = at::empty_like(q, at::MemoryFormat::Contiguous);
  seqs[0].out = out.data_ptr();
  run_attention(seqs, q, q.size(1), hkv, q.size(3), q.size(2), bits, scale, false);
  return out;
}

Tensor prefill(const Tensor &q, const Tensor &kd, const Tensor &km, const Tensor &vd,
               const Tensor &vm, const Tensor &rk, const Tensor &rv, int64_t packed,
               int64_t length, int64_t bits, double scale);

// Routes of the guarded entry points.
enum Route : int64_t { kDecode = 0, kVerify = 1, kPrefill = 2 };

using OptTensor = std::optional<Tensor>;

// Whether a kernel of this library covers the call; when it does not, the
// guarded op returns None and the caller falls back to dequantize + SDPA.
// The acceptance rules are those of the reference's guards -- one query:
// models/compressed_kv_attention.py:8-29; a chunk of 16..4096 queries with
// the bank shapes checked too: models/compressed_prefill_attention.py:6-52 --
// plus the verify route's limit of 16 query rows per KV head.  They are
// checked in the order the kernel touches the data: autograd state, the
// query, the presence of every cache tensor, the exact window, the banks.
bool covers(Route route, const Tensor &q, const OptTensor *view, int64_t packed, int64_t length,
            int64_t bits, double scale) {
  if (!q.is_cuda() || at::GradMode::is_enabled() || at::autocast::is_autocast_enabled(at::kCUDA) ||
      q.requires_grad())
    return false;
  if (q.dim() != 4 || q.size(0) != 1 || q.stride(3) != 1) return false;
  const auto dt = q.scalar_type();
  const int64_t n = q.size(2), d = q.size(3), hq = q.size(1);
  if ((dt != at::kBFloat16 && dt != at::kHalf) || (d != 64 && d != 128 && d != 256)) return false;
  if (!std::isfinite(scale) || (bits != 4 && bits != 8)) return false;
  const bool chunk = route == kPrefill;
  if (chunk ? (n < 16 || n > 4096) : (route == kDecode ? n != 1 : n < 1)) return false;
  if (packed < (chunk ? 1 : 128) || packed % 128) return false;
  for (int i = 0; i < 6; ++i) {
    const OptTensor &t = view[i];
    if (!t.has_value() || !t->defined() || t->device() != q.device() || t->requires_grad())
      return false;
  }
  // The exact window: [1,H,R,D] in the query dtype, rows dense, and long
  // enough to hold every query position.
  const Tensor &keys = *view[4], &values = *view[5];
  if (keys.dim() != 4 || values.sizes() != keys.sizes() || keys.size(0) != 1) return false;
  const int64_t h = keys.size(1), r = keys.size(2);
  if (h < 1 || hq < 1 || hq % h || hq / h > 16 || keys.size(3) != d) return false;
  if (keys.scalar_type() != dt || values.scalar_type() != dt) return false;
  if (keys.stride(3) != 1 || values.stride(3) != 1 || length != packed + r) return false;
  if (route != kDecode && r < n) return false;
  if (route == kVerify && n * (hq / h) > 16) return false;
  if (!chunk) return true;
  // The banks, [1,H,rows,...]: key codes (D, 128*bits/8) and meta (D, 2) per
  // 128-token unit; value codes (D/64, 64*bits/8) and meta (D/64, 2) per token.
  const Tensor &kd = *view[0], &km = *view[1], &vd = *view[2], &vm = *view[3];
  const int64_t per = 8 / bits;
  struct Want { const Tensor *t; at::ScalarType type; int64_t rows, a, b; };
  const Want want[4] = {{&kd, at::kByte, packed / 128, d, 128 / per},
                        {&km, at::kFloat, packed / 128, d, 2},
                        {&vd, at::kByte, packed, d / 64, 64 / per},
                        {&vm, at::kFloat, packed, d / 64, 2}};
  for (const Want &w : want) {
    const Tensor &t = *w.t;
    if (t.dim() != 5 || t.scalar_type() != w.type || t.size(0) != 1 || t.size(1) != h ||
        t.size(2) < w.rows || t.size(3) != w.a || t.size(4) != w.b || t.stride(4) != 1)
      return false;
  }
  return true;
}

// One call for the guard and the kernel: None when `covers` says no, else
// the route's output.
OptTensor attention_guarded(const Tensor &q, const OptTensor &kd, const OptTensor &km,
                            const OptTensor &vd, const OptTensor &vm, const OptTensor &rk,
                            const OptTensor &rv, int64_t packed, int64_t length, int64_t bits,
                            double scale, int64_t route) {
  const OptTensor view[6] = {kd, km, vd, vm, rk, rv};
  TORCH_CHECK(route >= kDecode && route <= kPrefill, "ckv::attention_guarded: unknown route ", route);
  if (!covers(Route(route), q, view, packed, length, bits, scale)) return std::nullopt;
  if (route == kPrefill) return prefill(q, *kd, *km, *vd, *vm, *rk, *rv, packed, length, bits, scale);
  return decode(q, *kd, *km, *vd, *vm, *rk, *rv, packed, length, bits, scale);
}

// The single-query route, the decode loop's entry (one argument fewer).
OptTensor decode_guarded(const Tensor &q, const OptTensor &kd, const OptTensor &km,
                         const OptTensor &vd, const OptTensor &vm, const OptTensor &rk,
                         const OptTensor &rv, int64_t packed, int64_t length, int64_t bits,
                         double scale) {
  return attention_guarded(q, kd, km, vd, vm, rk, rv, packed, length, bits, scale, kDecode);
}

// Packed prefill over one sequence's whole history
// (models/compressed_prefill_kernels.py:98-111): out [1,Hq,qlen,D] dense.
Tensor prefill(const Tensor &q, const Tensor &kd, const Tensor &km, const Tensor &vd,
               const Tensor &vm, const Tensor &rk, const Tensor &rv, int64_t packed,
               int64_t length, int64_t bits, double scale) {
  require_cuda(q, "query");
  TORCH_CHECK(q.dim() == 4 && q.size(0) == 1 && q.stride(3) == 1,
              "ckv::prefill: query must be [1,Hq,qlen,D] with a dense last dim");
  for (const Tensor *t : {&kd, &km, &vd, &vm, &rk, &rv})
    TORCH_CHECK(t->defined() && t->device() == q.device(),
                "ckv::prefill: all tensors must be on the query's device");
  TORCH_CHECK(packed >= 128 && packed % 128 == 0, "ckv::prefill: packed must be a positive multiple of 128");
  c10::cuda::CUDAGuard guard(q.device());
  const int64_t range[4] = {0, packed / 128, 0, rk.size(2)};
  const int64_t hkv = rk.size(1);
  const Tensor q2 = fit_rows(q);
  const Tensor kd2 = fit_bank(kd, 2), km2 = fit_bank(km, 2), vd2 = fit_bank(vd, 3),
               vm2 = fit_bank(vm, 3), rk2 = fit_rows(rk), rv2 = fit_rows(rv);
  ckv_prefill_args a{};
  a.seq = make_seq(q2, kd2, km2, vd2, vm2, rk2, rv2, packed, length, range, bits, hkv);
  Tensor out = at::empty(q.sizes(), q.options().memory_format(at::MemoryFormat::Contiguous));
  a.seq.out = out.data_ptr();
  a.heads_q = int32_t(q.size(1));
  a.heads_kv = int32_t(hkv);
  a.head_dim = int32_t(q.size(3));
  a.qlen = int32_t(q.size(2));
  a.bits = int32_t(bits);
  a.dtype = dtype_code(q.scalar_type());
  a.scale = float(scale);
  size_t bytes = 0;
  check_status(ckv_prefill_workspace(&a, &bytes), "prefill_workspace");
  Tensor ws;
  if (bytes)
    ws = at::empty({int64_t((bytes + 3) / 4)}, q.options().dtype(at::kFloat));
  check_status(ckv_prefill(&a, bytes ? ws.data_ptr() : nullptr, bytes, current_stream(q)), "prefill");
  return out;
}

Tensor combine_partials(const Tensor &partials, at::ScalarType dtype) {
  require_cuda(partials, "partials");
  TORCH_CHECK(partials.dim() == 3 && partials.scalar_type() == at::kFloat,
              "ckv::combine_partials: partials must be float32 [parts, rows, D+2]");
  c10::cuda::CUDAGuard guard(partials.device());
  Tensor p = partials.contiguous();
  const int64_t parts = p.size(0), rows = p.size(1), D = p.size(2) - 2;
  Tensor out = at::empty({rows, D}, p.options().dtype(dtype));
  check_status(ckv_combine_partials(p.data_ptr<float>(), int(parts), rows, int(D), dtype_code(dtype),
                                    out.data_ptr(), current_stream(p)),
               "combine_partials");
  return out;
}

// One rank's step of the peer exchange (ckv_exchange_combine): partial
// [rows, D+2] fp32 published to every rank's buffer, then the merged
// [rows, D] output (left unwritten when phases is 1, publish only).
Tensor exchange_combine(const Tensor &partial, std::vector<int64_t> buffers, int64_t rank,
                        int64_t phases, int64_t spin_limit, at::ScalarType dtype) {
  require_cuda(partial, "partial");
  TORCH_CHECK(partial.dim() == 2 && partial.scalar_type() == at::kFloat && partial.is_contiguous(),
              "ckv::exchange_combine: partial must be contiguous float32 [rows, D+2]");
  TORCH_CHECK(!buffers.empty() && buffers.size() <= CKV_EXCHANGE_MAX_WORLD,
              "ckv::exchange_combine: 1..", CKV_EXCHANGE_MAX_WORLD, " buffers");
  c10::cuda::CUDAGuard guard(partial.device());
  const int64_t rows = partial.size(0), D = partial.size(1) - 2;
  Tensor out = at::empty({rows, D}, partial.options().dtype(dtype));
  void *bufs[CKV_EXCHANGE_MAX_WORLD];
  for (size_t i = 0; i < buffers.size(); ++i) bufs[i] = reinterpret_cast<void *>(buffers[i]);
  check_status(ckv_exchange_combine(partial.data_ptr<float>(), rows, int(D), bufs, int(buffers.size()),
                                    int(rank), int(phases), spin_limit, dtype_code(dtype),
                                    out.data_ptr(), current_stream(partial)),
               "exchange_combine");
  return out;
}

// Error word of every cached attention workspace on `like`'s device (1 when
// a kernel gave up waiting for a copy or a peer warp and aborted, so that
// call's outputs are not valid).  Reading waits for each stream; the words
// are cleared afterwards.
int64_t attention_error(const Tensor &like) {
  TORCH_CHECK(like.is_cuda(), "ckv::attention_error: a CUDA tensor names the device");
  const int dev = int(like.get_device());
  auto &ws = workspaces();
  std::lock_guard<std::mutex> lock(ws.mu);
  int64_t any = 0;
  for (auto &kv : ws.buffers) {
    if (kv.first.first != dev) continue;
    int flag = 0;
    check_status(ckv_attention_error(kv.second.data_ptr(), &flag,
                                     reinterpret_cast<ckv_stream_t>(kv.first.second)),
                 "attention_error");
    if (flag) {
      C10_CUDA_CHECK(cudaMemsetAsync(kv.second.data_ptr(), 0, 4, kv.first.second));
      C10_CUDA_CHECK(cudaStreamSynchronize(kv.first.second));
      any = 1;
    }
  }
  return any;
}

}  // namespace

TORCH_LIBRARY(ckv, m) {
  m.def("pack_rows(Tensor rows, int bits, int rounding) -> (Tensor, Tensor)");
  m.def("unpack_rows(Tensor data, Tensor meta, int bits, ScalarType dtype) -> Tensor");
  m.def(
      "pack_append(Tensor keys, Tensor values, Tensor(a!) key_data, Tensor(b!) key_meta, "
      "Tensor(c!) value_data, Tensor(d!) value_meta, int count, int unit_offset, int bits, "
      "int rounding) -> ()");
  m.def(
      "attention(Tensor[] queries, Tensor?[] key_data, Tensor?[] key_meta, Tensor?[] value_data, "
      "Tensor?[] value_meta, Tensor?[] keys, Tensor?[] values, int[] packed, int[] lengths, "
      "int[] ranges, int bits, float scale, bool partial) -> Tensor[]");
  m.def("combine_partials(Tensor partials, ScalarType dtype) -> Tensor");
  m.def(
      "decode(Tensor query, Tensor key_data, Tensor key_meta, Tensor value_data, Tensor value_meta, "
      "Tensor keys, Tensor values, int packed, int length, int bits, float scale) -> Tensor");
  m.def("attention_error(Tensor like) -> int");
  m.def(
      "prefill(Tensor query, Tensor key_data, Tensor key_meta, Tensor value_data, Tensor value_meta, "
      "Tensor keys, Tensor values, int packed, int length, int bits, float scale) -> Tensor");
  // Any device (a CPU query gets None), so a catch-all kernel.
  m.def(
      "decode_guarded(Tensor query, Tensor? key_data, Tensor? key_meta, Tensor? value_data, "
      "Tensor? value_meta, Tensor? keys, Tensor? values, int packed, int length, int bits, "
      "float scale) -> Tensor?",
      &decode_guarded);
  m.def(
      "attention_guarded(Tensor query, Tensor? key_data, Tensor? key_meta, Tensor? value_data, "
      "Tensor? value_meta, Tensor? keys, Tensor? values, int packed, int length, int bits, "
      "float scale, int route) -> Tensor?",
      &attention_guarded);
  m.def("residual_append(Tensor keys_new, Tensor values_new, Tensor(a!) keys, Tensor(b!) values, "
        "int offset) -> (Tensor(a), Tensor(b))");
  m.def("window_append(Tensor keys_new, Tensor values_new, Tensor(a!) keys, Tensor(b!) values, "
        "int capacity) -> (Tensor(a), Tensor(b))");
  m.def("set_dequant(int mode) -> int", &set_dequant);
  m.def("exchange_combine(Tensor partial, int[] buffers, int rank, int phases, int spin_limit, "
        "ScalarType dtype) -> Tensor");
}

namespace {
std::vector<Tensor> attention_opt(const std::vector<Tensor> &queries,
                                  const c10::List<std::optional<Tensor>> &kd,
                                  const c10::List<std::optional<Tensor>> &km,
                                  const c10::List<std::optional<Tensor>> &vd,
                                  const c10::List<std::optional<Tensor>> &vm,
                                  const c10::List<std::optional<Tensor>> &rk,
                                  const c10::List<std::optional<Tensor>> &rv,
                                  std::vector<int64_t> packed, std::vector<int64_t> lengths,
                                  std::vector<int64_t> ranges, int64_t bits, double scale,
                                  bool partial) {
  auto unwrap = [](const c10::List<std::optional<Tensor>> &l) {
    std::vector<Tensor> v;
    v.reserve(l.size());
    for (size_t i = 0; i < l.size(); ++i) {
      std::optional<Tensor> t = l.get(i);
      v.push_back(t.has_value() ? *t : Tensor());
    }
    return v;
  };
  return attention(queries, unwrap(kd), unwrap(km), unwrap(vd), unwrap(vm), unwrap(rk), unwrap(rv),
                   std::move(packed), std::move(lengths), std::move(ranges), bits, scale, partial);
}
}  // namespace

TORCH_LIBRARY_IMPL(ckv, CUDA, m) {
  m.impl("pack_rows", &pack_rows);
  m.impl("unpack_rows", &unpack_rows);
  m.impl("pack_append", &pack_append);
  m.impl("attention", &attention_opt);
  m.impl("combine_partials", &combine_partials);
  m.impl("exchange_combine", &exchange_combine);
  m.impl("decode", &decode);
  m.impl("attention_error", &attention_error);
  m.impl("residual_append", &residual_append);
  m.impl("window_append", &window_append);
  m.impl("prefill", &prefill);
}
