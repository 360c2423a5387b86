"""Route the reference's kernel modules to the B200 kernels.

``install()`` makes ``models.quantized_kv_kernels``,
``models.compressed_kv_kernels`` and ``models.compressed_prefill_kernels``
resolve to ``trpg_b200``'s modules, so the reference's own cache
(``models/quantized_kv.py:16-18,29-31``), guards
(``models/compressed_kv_attention.py:25-28``,
``models/compressed_prefill_attention.py:46-51``) and every caller above them
(``cached_generation``, ``mtp_generation``, ``cuda_graph_decode``) run on
these kernels without edits.  ``uninstall()`` restores whatever was there.
"""
from __future__ import annotations

import sys

_saved: dict[str, object] = {}


def install(package: str = 'models') -> None:
    from . import _native, compressed_kv_kernels, compressed_prefill_kernels, quantized_kv_kernels
    _native.load()   # fail here, loudly, if the libraries are not built
    for name, module in (('quantized_kv_kernels', quantized_kv_kernels),
                         ('compressed_kv_kernels', compressed_kv_kernels),
                         ('compressed_prefill_kernels', compressed_prefill_kernels)):
        full = f'{package}.{name}'
        _saved.setdefault(full, sys.modules.get(full))
        sys.modules[full] = module
        parent = sys.modules.get(package)
        if parent is not None:
            setattr(parent, name, module)


def uninstall(package: str = 'models') -> None:
    for name in ('quantized_kv_kernels', 'compressed_kv_kernels', 'compressed_prefill_kernels'):
        full = f'{package}.{name}'
        if full not in _saved:
            continue
        old = _saved.pop(full)
        if old is None:
            sys.modules.pop(full, None)
        else:
            sys.modules[full] = old
