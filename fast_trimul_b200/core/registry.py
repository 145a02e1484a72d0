"""Plug-in tables, same API as the reference's fast_trimul/core/registry.py:12-56:
`@backend(name, **caps)` registers a backend instance, `@weights_for(source)`
registers a state_dict remap."""

from .context import BackendCapabilities

_BACKENDS: dict = {}
_LOADERS: dict = {}


def backend(name: str, **capabilities):
    def register(cls):
        _BACKENDS[name] = cls(BackendCapabilities(**capabilities))
        return cls
    return register


def get_backend(name: str):
    return _BACKENDS.get(name)


def list_backends() -> list:
    return list(_BACKENDS)


def weights_for(source: str):
    def register(fn):
        _LOADERS[source] = fn
        return fn
    return register


def get_loader(source: str):
    try:
        return _LOADERS[source]
    except KeyError:
        raise KeyError(f"no weight loader registered for {source!r} "
                       f"(available: {sorted(_LOADERS)})") from None
