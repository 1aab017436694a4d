"""A numpy stand-in for the small slice of ``jax.numpy`` that the reference EAM/LJ math uses.

Fixture-generation infrastructure only: ``make_golden.py`` installs this module as ``jax`` /
``jax.numpy`` so that the reference's own ``lammps_jax/eam.py`` (and the LJ energy builder in
``examples/export_model.py``) execute unchanged on numpy arrays in this container, where jax is
not installed. No autodiff is provided; fixtures take forces from the reference's analytic
per-edge force builder (``make_setfl_edge_force``) and check them against central differences
of the reference energy.

Covered API: ``asarray``, ``zeros``, ``clip``, ``floor``, ``minimum``, ``maximum``, ``where``,
``sqrt``, ``sum``, dtype names, and ``x.at[idx].get/add/set`` with a ``mode`` keyword that is
accepted and ignored (indices in the fixtures are always in bounds).
"""

import sys
import types

import numpy as np


class Array(np.ndarray):
    """ndarray subclass carrying jax's functional ``.at[...]`` indexer."""

    @property
    def at(self):
        return _AtIndexer(self)


class _AtIndexer:
    def __init__(self, base):
        self._base = base

    def __getitem__(self, index):
        return _AtRef(self._base, index)


class _AtRef:
    def __init__(self, base, index):
        self._base = base
        self._index = _plain(index)

    def get(self, mode=None):
        del mode
        return wrap(np.asarray(self._base)[self._index])

    def add(self, values, mode=None):
        del mode
        out = np.array(self._base, copy=True)
        np.add.at(out, self._index, np.asarray(values, dtype=out.dtype))
        return wrap(out)

    def set(self, values, mode=None):
        del mode
        out = np.array(self._base, copy=True)
        out[self._index] = np.asarray(values, dtype=out.dtype)
        return wrap(out)


def _plain(index):
    if isinstance(index, tuple):
        return tuple(_plain(i) for i in index)
    if isinstance(index, np.ndarray):
        return np.asarray(index)
    return index


def wrap(value):
    return np.asarray(value).view(Array)


def asarray(value, dtype=None):
    return wrap(np.asarray(value, dtype=dtype))


def zeros(shape, dtype=None):
    return wrap(np.zeros(shape, dtype=dtype))


def _ufunc(fn):
    def call(*args, **kwargs):
        return wrap(fn(*[np.asarray(a) if isinstance(a, np.ndarray) else a for a in args],
                       **kwargs))
    return call


def make_module():
    """Build fake ``jax`` and ``jax.numpy`` modules backed by this file."""
    jnp = types.ModuleType("jax.numpy")
    jnp.asarray = asarray
    jnp.array = asarray
    jnp.zeros = zeros
    for name in ("clip", "floor", "minimum", "maximum", "where", "sqrt", "sum", "exp",
                 "abs", "any", "arange", "ones"):
        setattr(jnp, name, _ufunc(getattr(np, name)))
    for name in ("int8", "int32", "int64", "float32", "float64", "bool_"):
        setattr(jnp, name, getattr(np, name))
    jax = types.ModuleType("jax")
    jax.numpy = jnp
    return jax, jnp


def install():
    """Register the fake modules; returns (jax, jnp)."""
    jax, jnp = make_module()
    sys.modules["jax"] = jax
    sys.modules["jax.numpy"] = jnp
    return jax, jnp
