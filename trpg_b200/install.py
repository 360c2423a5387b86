"""Route the reference's compressed-KV modules to this package.

``install()`` makes every module of the path resolve to ``trpg_b200``'s
mirror of it:

==================================  =====================================
reference module                    replaced by
==================================  =====================================
``models.quantized_kv_kernels``     ``trpg_b200.quantized_kv_kernels``
``models.compressed_kv_kernels``    ``trpg_b200.compressed_kv_kernels``
``models.compressed_prefill_kernels`` ``trpg_b200.compressed_prefill_kernels``
``models.quantized_kv``             ``trpg_b200.quantized_kv`` (the cache:
                                    direct-to-slab append, in-place window)
``models.compressed_kv_attention``  ``trpg_b200.compressed_kv_attention``
                                    (the model patch: decode, verify and
                                    prefill routing)
``models.compressed_prefill_attention`` ``trpg_b200.compressed_prefill_attention``
``models.mtp_verification_kernels`` ``trpg_b200.mtp_verification_kernels``
==================================  =====================================

The reference's callers bind these names at import time
(``models/cached_generation.py:4``, ``models/mtp_generation.py:15-17``,
``models/hybrid_cache_transaction.py:16``, ``models/prefix_cache.py:6``,
``models/pretrained.py:133-138``).  Modules imported after ``install()``
get this package's objects through ``sys.modules``; modules of the package
that were imported before it have each name that referred to a replaced
module's object re-pointed at this package's object of the same name.  If
the reference's verify-scope module was loaded first, this package adopts
its flag, so a scope entered through either module is seen.

``uninstall()`` restores the module table (names re-pointed in loaded
modules stay re-pointed).
"""
from __future__ import annotations

import sys

MODULES = ('quantized_kv_kernels', 'compressed_kv_kernels', 'compressed_prefill_kernels',
           'quantized_kv', 'compressed_kv_attention', 'compressed_prefill_attention',
           'mtp_verification_kernels')

_saved: dict[str, object] = {}


def _ours(name):
    import importlib
    return importlib.import_module(f'{__package__}.{name}')


def install(package: str = 'models') -> None:
    from . import _native
    _native.load()   # fail here, loudly, if the libraries are not built
    ours = {name: _ours(name) for name in MODULES}
    theirs = {}
    for name in MODULES:
        full = f'{package}.{name}'
        old = sys.modules.get(full)
        _saved.setdefault(full, old)
        if old is not None and old is not ours[name]:
            theirs[name] = old
    old_scope = theirs.get('mtp_verification_kernels')
    flag = getattr(old_scope, '_MTP_VERIFICATION_ENABLED', None)
    if flag is not None:
        ours['mtp_verification_kernels'].bind(flag)
    for name in MODULES:
        sys.modules[f'{package}.{name}'] = ours[name]
        parent = sys.modules.get(package)
        if parent is not None:
            setattr(parent, name, ours[name])
    # Functions and classes the package's loaded modules imported by name
    # from a replaced module (``from .quantized_kv import make_cache``).
    prefix = package + '.'
    for mod_name, module in list(sys.modules.items()):
        if not mod_name.startswith(prefix) or module is None:
            continue
        if any(module is m for m in ours.values()) or any(module is m for m in theirs.values()):
            continue
        for attr, value in list(vars(module).items()):
            if attr.startswith('__') or not callable(value):
                continue
            for name, old in theirs.items():
                if getattr(old, attr, None) is value and hasattr(ours[name], attr):
                    setattr(module, attr, getattr(ours[name], attr))
                    break


def uninstall(package: str = 'models') -> None:
    for name in MODULES:
        full = f'{package}.{name}'
        if full not in _saved:
            continue
        old = _saved.pop(full)
        if old is None:
            sys.modules.pop(full, None)
        else:
            sys.modules[full] = old
