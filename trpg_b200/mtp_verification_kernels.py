"""Request-local opt-in for multi-query (MTP) verification kernels.

Same interface as ``models/mtp_verification_kernels.py:11-25``: a flag that
nested scopes, exceptions and independent threads/tasks each keep for
themselves, read by ``compressed_kv_attention._forward`` to route 2..4-query
calls to the verify kernel.

There must be one flag, not two: the reference's MTP loop
(``models/mtp_generation.py:15,86``) enters the scope of whatever module it
imported.  ``trpg_b200.install`` therefore maps the reference module name to
this module, and, when the reference module was imported before that,
``bind()`` adopts its flag object, so that the scope functions of both
modules set the flag this package reads.
"""
from contextlib import contextmanager
from contextvars import ContextVar

_MTP_VERIFICATION_ENABLED = ContextVar('mtp_verification_kernels_enabled', default=False)


def bind(flag: ContextVar) -> None:
    """Use ``flag`` (the reference module's ContextVar) as this module's flag."""
    global _MTP_VERIFICATION_ENABLED
    if not isinstance(flag, ContextVar):
        raise TypeError('expected the ContextVar of the reference scope module')
    _MTP_VERIFICATION_ENABLED = flag


def mtp_verification_enabled():
    return _MTP_VERIFICATION_ENABLED.get()


@contextmanager
def mtp_verification_scope(enabled=True):
    flag = _MTP_VERIFICATION_ENABLED
    token = flag.set(bool(enabled))
    try:
        yield
    finally:
        flag.reset(token)
