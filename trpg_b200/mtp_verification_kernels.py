"""Request-local opt-in for multi-query (MTP) verification kernels.

Mirror of ``models/mtp_verification_kernels.py:11-25``: a ContextVar flag
that nested scopes, exceptions and independent threads/tasks each keep for
themselves.  ``compressed_kv_attention._forward`` routes 2..4-query calls to
the compressed-KV verify kernel only inside this scope.
"""
from contextlib import contextmanager
from contextvars import ContextVar

_MTP_VERIFICATION_ENABLED = ContextVar('mtp_verification_kernels_enabled', default=False)


def mtp_verification_enabled():
    return _MTP_VERIFICATION_ENABLED.get()


@contextmanager
def mtp_verification_scope(enabled=True):
    token = _MTP_VERIFICATION_ENABLED.set(bool(enabled))
    try:
        yield
    finally:
        _MTP_VERIFICATION_ENABLED.reset(token)
