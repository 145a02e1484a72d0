"""Scoped backend preference, same API as fast_trimul/core/decorators.py:15-45:
a ContextVar (thread- and task-local) set by `accelerated(...)` / `@accelerate`."""

import contextlib
import functools
from contextvars import ContextVar

_ACTIVE_BACKEND: ContextVar = ContextVar("fast_trimul_b200_backend", default="auto")


def active_backend() -> str:
    return _ACTIVE_BACKEND.get()


@contextlib.contextmanager
def accelerated(backend: str = "auto"):
    token = _ACTIVE_BACKEND.set(backend)
    try:
        yield
    finally:
        _ACTIVE_BACKEND.reset(token)


def accelerate(func=None, *, backend: str = "auto"):
    def wrap(fn):
        @functools.wraps(fn)
        def inner(*args, **kwargs):
            with accelerated(backend):
                return fn(*args, **kwargs)
        return inner
    return wrap(func) if callable(func) else wrap
