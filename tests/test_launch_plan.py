"""Launch plan of ``ckv_attention`` through the C ABI, without a GPU.

``ckv_attention_workspace`` validates the arguments and plans the launch but
reads no tensor memory, so fake (aligned, non-null) addresses are enough.
The byte count it returns holds the grid size: a 256-byte header, one
4-byte ticket per (sequence, KV head) slot (64 x 128 slots), then per CTA a
[rows][D] fp32 record and a 16-byte-padded (m, l) record, each array
rounded to 256 bytes (trpg_b200/csrc/ckv_attn.cu).  Without a device the
plan assumes 148 SMs, the B200's count.
"""
import ctypes

from tests.test_zz_no_alloc import AttnArgs, Seq, _lib

SMS = 148
HEADER = 256 + 64 * 128 * 4


def _grid(nbytes, rows, dim):
    mls = (rows * 2 + 3) & ~3
    r256 = lambda x: (x + 255) // 256 * 256
    for g in range(1, 1 << 16):
        if HEADER + r256(g * rows * dim * 4) + r256(g * mls * 4) == nbytes:
            return g
    raise AssertionError(f'no grid gives {nbytes} bytes')


def _plan(lengths, nq=1, hq=16, hkv=4, dim=256, resid=256):
    seqs = []
    for i, length in enumerate(lengths):
        packed = (length - resid) // 128 * 128
        base = 0x100000 * (i + 1)
        seqs.append(Seq(base, 0, dim, base, 32768, 32768, base, 512, 512, base, 256, 256,
                        base, 8, 8, base, 8 * dim, dim, base, 8 * dim, dim,
                        packed, length, 0, packed // 128, 0, length - packed, base))
    arr = (Seq * len(seqs))(*seqs)
    args = AttnArgs(arr, len(seqs), hq, hkv, dim, nq, 8, 0, 0.0625, 0, 0)
    nbytes = ctypes.c_size_t()
    assert _lib().ckv_attention_workspace(ctypes.byref(args), ctypes.byref(nbytes)) == 0
    return _grid(nbytes.value, nq * hq // hkv, dim)


def test_one_long_sequence_is_one_wave():
    # 4 pairs: each gets at least 8 CTAs, so one wave whatever the length.
    assert _plan([32768]) == SMS
    assert _plan([131072]) == SMS


def test_many_pairs_fill_whole_waves_exactly():
    # 16 x 4 pairs of 130 items with 16 query rows (32 items a CTA): 2 waves
    # of about 28 items, rounded by largest remainders to exactly 2 x 148
    # CTAs (not 64 x 5 = 320).
    assert _plan([16384] * 16, nq=4) == 2 * SMS
    # 4 query rows (24 items a CTA): whole waves as well.
    ragged = [1024 + (i * 1777) % 7169 for i in range(64)]
    packed = [(n - 256) // 128 * 128 for n in ragged]
    total = sum(p // 128 + -(-(n - p) // 64) for n, p in zip(ragged, packed)) * 4
    assert _plan(ragged) == -(-total // (SMS * 24)) * SMS
