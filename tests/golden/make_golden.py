"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run in a container that has the reference source tree (read-only is fine):

    python tests/golden/make_golden.py /path/to/reference

It imports the reference's own modules and records what they compute:

* ``quantizer.npz``  -- ``models/quantized_kv.py:_pack`` (CPU, round half to
  even) and ``models/quantized_kv_kernels.py:pack`` (the Triton kernel, run by
  the Triton interpreter on CPU tensors, round half up) on seeded rows,
  including tie-heavy, constant, tiny-range and outlier rows; plus
  ``_unpack`` (CPU, separate multiply and add) of the CPU codes.
* ``attention.npz``  -- cache states built with ``QuantizedAttentionLayer``
  (``update`` then ``append_for_attention``, as in
  ``scripts/profile_compressed_kv.py:31-36``) and the reference oracle output
  ``scaled_dot_product_attention(q, cat(unpack, residual), enable_gqa=True)``
  (with ``causal_lower_right`` for multi-query cases), plus sha256 digests of
  the packed banks and residual windows.

Inputs come from ``oracle.ckv_oracle.seeded_normal`` so the tests regenerate
them without the reference.  Nothing here runs on the GPU box.
"""
import os
import sys
from pathlib import Path

os.environ['TRITON_INTERPRET'] = '1'          # run the Triton pack on CPU tensors

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

import numpy as np  # noqa: E402

from oracle import ckv_oracle as O  # noqa: E402

# (name, bits, heads_kv, heads_q, length, dim, new_tokens, dtype, seed, scale, outliers)
ATTENTION_CASES = [
    ('c1_q8_l2048', 8, 4, 16, 2048, 256, 1, 'bfloat16', 1, 1 / 16, False),
    ('q4_l2048', 4, 4, 16, 2048, 256, 1, 'bfloat16', 11, 1 / 16, False),
    ('q8_fp16_l1000_d128', 8, 2, 6, 1000, 128, 1, 'float16', 12, 128 ** -0.5, False),
    ('q4_l4097_d64_gqa3', 4, 2, 6, 4097, 64, 1, 'bfloat16', 13, 64 ** -0.5, False),
    ('q8_outliers_l3000', 8, 4, 16, 3000, 256, 1, 'bfloat16', 14, 1 / 16, True),
    ('verify_q8_n4_l1500', 8, 4, 16, 1500, 256, 4, 'bfloat16', 15, 1 / 16, False),
    ('verify_q4_n2_l700', 4, 4, 16, 700, 256, 2, 'bfloat16', 16, 1 / 16, False),
    ('verify_q8_n3_l2000_d128', 8, 2, 8, 2000, 128, 3, 'float16', 17, 128 ** -0.5, False),
]


def quantizer_rows(seed, group, count=192):
    """Seeded rows plus hand-made edge rows for one group size."""
    rows = [O.seeded_normal(seed, (count, group))]
    tie = np.zeros((8, group), np.float32)
    tie[:, 1::2] = 1.0                                       # exact half-code ties
    tie[:, ::4] = -1.0
    rows.append(O.round_to(tie * np.linspace(1, 4, 8, dtype=np.float32)[:, None], 'bfloat16'))
    rows.append(np.full((4, group), 0.75, np.float32))       # constant -> scale clamp
    rows.append(O.round_to(O.seeded_normal(seed + 1, (8, group)) * 1e-6, 'bfloat16'))
    rows.append(O.round_to(O.seeded_normal(seed + 2, (8, group)) * 8, 'bfloat16'))
    ramp = np.arange(group, dtype=np.float32)[None, :] * np.float32(0.25) - 3
    rows.append(O.round_to(np.repeat(ramp, 4, 0), 'bfloat16'))
    return np.concatenate(rows).astype(np.float32)


def main(reference: str):
    sys.path.insert(0, reference)
    import torch
    from torch.nn import functional as F
    from torch.nn.attention.bias import causal_lower_right
    from models.quantized_kv import QuantizedAttentionLayer, _pack, _unpack
    from models.quantized_kv_kernels import pack as triton_pack

    out = {}
    for bits in (8, 4):
        for group, seed in ((128, 101), (64, 102)):
            rows = quantizer_rows(seed + bits, group)
            t = torch.from_numpy(rows).bfloat16()
            codes, meta = _pack(t, bits)
            tcodes, tmeta = triton_pack(t.contiguous(), bits)
            deq = _unpack(codes, meta, bits, torch.bfloat16).float().numpy()
            key = f'b{bits}_g{group}'
            out[f'{key}_rows'] = rows
            out[f'{key}_cpu_codes'] = codes.numpy()
            out[f'{key}_cpu_meta'] = meta.numpy()
            out[f'{key}_triton_codes'] = tcodes.numpy()
            out[f'{key}_triton_meta'] = tmeta.numpy()
            out[f'{key}_cpu_unpack_bf16'] = deq
    np.savez_compressed(HERE / 'quantizer.npz', **out)

    att = {}
    for name, bits, hkv, hq, length, dim, n, dtype, seed, scale, outliers in ATTENTION_CASES:
        tdt = dict(bfloat16=torch.bfloat16, float16=torch.float16)[dtype]
        _, k, v = O.cache_state(seed, hkv, length, dim, bits, n, dtype, outliers=outliers)
        q = O.seeded_normal(seed + 2, (1, hq, n, dim), dtype)
        kt, vt = torch.from_numpy(k).to(tdt), torch.from_numpy(v).to(tdt)
        layer = QuantizedAttentionLayer(bits)
        with torch.inference_mode():
            layer.update(kt[:, :, :length - n], vt[:, :, :length - n])
            view = layer.append_for_attention(kt[:, :, length - n:], vt[:, :, length - n:])
            keys = torch.cat((layer.key_bank.unpack(tdt), view.keys), -2)
            values = torch.cat((layer.value_bank.unpack(tdt), view.values), -2)
            mask = causal_lower_right(n, view.length) if n > 1 else None
            expected = F.scaled_dot_product_attention(torch.from_numpy(q).to(tdt), keys, values,
                                                      attn_mask=mask, enable_gqa=True, scale=scale)
        units = layer.key_bank.units
        att[f'{name}_spec'] = np.array([bits, hkv, hq, length, dim, n, seed, int(outliers)], np.int64)
        att[f'{name}_dtype'] = np.array(dtype)
        att[f'{name}_scale'] = np.array(scale, np.float64)
        att[f'{name}_packed'] = np.array(view.packed_tokens, np.int64)
        att[f'{name}_residual'] = np.array(view.keys.shape[2], np.int64)
        att[f'{name}_bank_digest'] = np.array(O.digest(
            layer.key_bank.data[:, :, :units].contiguous().numpy(),
            layer.key_bank.meta[:, :, :units].contiguous().numpy(),
            layer.value_bank.data[:, :, :units * 128].contiguous().numpy(),
            layer.value_bank.meta[:, :, :units * 128].contiguous().numpy()))
        att[f'{name}_residual_digest'] = np.array(O.digest(
            view.keys.float().numpy(), view.values.float().numpy()))
        att[f'{name}_output'] = expected.float().numpy()
        print(name, 'packed', view.packed_tokens, 'residual', view.keys.shape[2])
    np.savez_compressed(HERE / 'attention.npz', **att)


if __name__ == '__main__':
    if len(sys.argv) != 2:
        sys.exit('usage: python tests/golden/make_golden.py REFERENCE_SOURCE_TREE')
    main(sys.argv[1])
