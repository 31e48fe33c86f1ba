"""A numpy stand-in for the parts of jax the reference package imports.

jax is not installable in this environment, so to obtain the reference's own
outputs, tests/golden/make_golden.py installs this module as ``jax`` (and
``jax.numpy``, ``jax.nn``, ``jax.lax``, ``jax.experimental.pallas`` and
``jax.experimental.pallas.triton``) before importing the reference source.

Pallas kernels run the way ``pallas_call(..., interpret=True)`` runs them: the
kernel body is called once per grid point with block views of its operands
selected by each BlockSpec's index map (block index times block shape); loads
copy a view, stores write through it.  ``pl.dot`` is an fp32 numpy matmul.
``jit`` and ``custom_vjp`` are transparent wrappers.
"""
from __future__ import annotations

import sys
import types

import numpy as np

_PROGRAM_ID = [0, 0, 0]


# ---------------------------------------------------------------- jax core
def jit(fun=None, **_kw):
    if fun is None:
        return lambda f: f
    return fun


class custom_vjp:  # noqa: N801 - mirrors jax.custom_vjp
    def __init__(self, fun, nondiff_argnums=()):
        self.fun = fun
        self.nondiff_argnums = nondiff_argnums
        self.fwd = self.bwd = None

    def defvjp(self, fwd, bwd):
        self.fwd, self.bwd = fwd, bwd

    def __call__(self, *args, **kwargs):
        return self.fun(*args, **kwargs)


class ShapeDtypeStruct:
    def __init__(self, shape, dtype):
        self.shape = tuple(shape)
        self.dtype = np.dtype(dtype)


def _softmax(x, axis=-1):
    e = np.exp(x - np.max(x, axis=axis, keepdims=True))
    return e / np.sum(e, axis=axis, keepdims=True)


def _fori_loop(lo, hi, body, init):
    val = init
    for i in range(int(lo), int(hi)):
        val = body(i, val)
    return val


# ---------------------------------------------------------------- pallas
class BlockSpec:
    def __init__(self, block_shape, index_map):
        self.block_shape = tuple(block_shape)
        self.index_map = index_map


class _Slice:
    def __init__(self, start, size):
        self.start, self.size = int(start), int(size)


def dslice(start, size):
    return _Slice(start, size)


def _conv(idx):
    if not isinstance(idx, tuple):
        idx = (idx,)
    return tuple(slice(i.start, i.start + i.size) if isinstance(i, _Slice) else i for i in idx)


class Ref:
    def __init__(self, view: np.ndarray):
        self.view = view

    @property
    def at(self):
        ref = self

        class _At:
            def __getitem__(self, idx):
                return Ref(ref.view[_conv(idx)])

        return _At()

    @property
    def shape(self):
        return self.view.shape

    @property
    def dtype(self):
        return self.view.dtype


def program_id(axis):
    return _PROGRAM_ID[axis]


def cdiv(a, b):
    return -(-a // b)


def dot(a, b, trans_a=False, trans_b=False, precision=None, **_kw):
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    return (a.T if trans_a else a) @ (b.T if trans_b else b)


def _block(arr, spec, gidx):
    bidx = spec.index_map(*gidx)
    return arr[tuple(slice(int(b) * s, int(b) * s + s) for b, s in zip(bidx, spec.block_shape))]


def pallas_call(kernel, out_shape, grid, in_specs, out_specs, interpret=False, compiler_params=None, **_kw):
    single = not isinstance(out_shape, (list, tuple))
    outs_sd = [out_shape] if single else list(out_shape)
    ospecs = [out_specs] if not isinstance(out_specs, (list, tuple)) else list(out_specs)

    def call(*args):
        outs = [np.zeros(s.shape, s.dtype) for s in outs_sd]
        for gidx in np.ndindex(*grid):
            _PROGRAM_ID[: len(gidx)] = gidx
            refs = [Ref(_block(np.asarray(a), sp, gidx)) for a, sp in zip(args, in_specs)]
            refs += [Ref(_block(o, sp, gidx)) for o, sp in zip(outs, ospecs)]
            kernel(*refs)
        return outs[0] if single else outs

    return call


def load(ref):
    return np.array(ref.view)


def store(ref, val):
    ref.view[...] = val


class CompilerParams:
    def __init__(self, **kw):
        self.kw = kw


# ---------------------------------------------------------------- module wiring
def install() -> None:
    jax = types.ModuleType("jax")
    jnp = types.ModuleType("jax.numpy")
    jnp.__getattr__ = lambda name: getattr(np, name)  # type: ignore[attr-defined]
    nn = types.ModuleType("jax.nn")
    nn.softmax = _softmax
    lax = types.ModuleType("jax.lax")
    lax.fori_loop = _fori_loop
    exp = types.ModuleType("jax.experimental")
    pl = types.ModuleType("jax.experimental.pallas")
    for name in ("BlockSpec", "program_id", "cdiv", "dot", "pallas_call", "dslice"):
        setattr(pl, name, globals()[name])
    tr = types.ModuleType("jax.experimental.pallas.triton")
    tr.load, tr.store, tr.CompilerParams = load, store, CompilerParams
    pl.triton = tr
    exp.pallas = pl
    jax.numpy, jax.nn, jax.lax, jax.experimental = jnp, nn, lax, exp
    jax.jit, jax.custom_vjp, jax.ShapeDtypeStruct, jax.Array = jit, custom_vjp, ShapeDtypeStruct, np.ndarray
    sys.modules.update({
        "jax": jax, "jax.numpy": jnp, "jax.nn": nn, "jax.lax": lax, "jax.experimental": exp,
        "jax.experimental.pallas": pl, "jax.experimental.pallas.triton": tr,
    })
