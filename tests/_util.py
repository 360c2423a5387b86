"""Shared helpers for the parity tests (inputs come from the oracle's seeded generator)."""
import numpy as np
import torch

from oracle import ckv_oracle as O

TORCH_DTYPE = {'bfloat16': torch.bfloat16, 'float16': torch.float16}


def to_torch(a: np.ndarray, dtype: str, device='cuda') -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(device).to(TORCH_DTYPE[dtype])


def gpu_cache_state(seed, heads, length, dim, bits, new_tokens=1, dtype='bfloat16',
                    outliers=False, rounding='half_even'):
    """Same reference-reachable state as ``O.cache_state``, built by the B200 cache.

    Returns (gpu_layer, gpu_view, oracle_layer).
    """
    from trpg_b200.quantized_kv import QuantizedAttentionLayer
    olayer, k, v = O.cache_state(seed, heads, length, dim, bits, new_tokens, dtype,
                                 rounding=rounding, outliers=outliers)
    kt, vt = to_torch(k, dtype), to_torch(v, dtype)
    layer = QuantizedAttentionLayer(bits, rounding)
    with torch.inference_mode():
        layer.update(kt[:, :, :length - new_tokens], vt[:, :, :length - new_tokens])
        view = layer.append_for_attention(kt[:, :, length - new_tokens:].contiguous(),
                                          vt[:, :, length - new_tokens:].contiguous())
    return layer, view, olayer


def bank_arrays(layer):
    """Used rows of the GPU banks as numpy arrays (oracle layout)."""
    u = layer.key_bank.units
    return (layer.key_bank.data[:, :, :u].cpu().numpy(), layer.key_bank.meta[:, :, :u].cpu().numpy(),
            layer.value_bank.data[:, :, :u * 128].cpu().numpy(),
            layer.value_bank.meta[:, :, :u * 128].cpu().numpy())


def residual_arrays(view):
    return view.keys.float().cpu().numpy(), view.values.float().cpu().numpy()


def max_abs(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))
