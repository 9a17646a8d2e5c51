"""A numpy stand-in for the few ``jax`` names the reference's source uses.

TEST INFRASTRUCTURE ONLY: ``make_reference_golden.py`` installs these modules
in ``sys.modules`` so that the UNMODIFIED reference files
(``src/pallas_flash/*.py`` and ``tests/test_paged.py`` of
aabhimittal/TPU-Native-Pallas-FlashAttention) can be executed in a container
without jax, to produce golden vectors.  Nothing here is shipped or timed.

What is restated (the published semantics of jax, pinned in the reference by
``jax>=0.4.30``, ``pyproject.toml:12-15``):

* ``jax.numpy``: numpy, with ``jnp.float32`` widened to float64 in the default
  ``WIDE`` mode so the golden outputs carry float64 accuracy; arrays support
  ``x.at[idx].set(v)`` (functional update).
* ``jax.lax``: ``broadcasted_iota``, ``rsqrt``, ``dynamic_update_slice`` and
  ``dynamic_update_slice_in_dim`` with jax's clamp rule (a start index is
  clamped to ``[0, dim - update_dim]``).
* ``jax.nn``: ``softmax`` (max-subtracted exp / sum) and ``silu``.
* ``jax.custom_vjp``: calling the primal function; the fwd/bwd rules are
  called by the generator directly.
* ``jax.experimental.pallas``: ``pallas_call`` executes the kernel body once
  per grid point in lexicographic grid order (the order Pallas interpret mode
  and the TPU use), with scratch buffers persisting across grid points, inputs
  sliced by each ``BlockSpec``'s index map (blocks that run past the array end
  are padded with NaN, the "uninitialised" fill of interpret mode), outputs
  written back block by block, and ``PrefetchScalarGridSpec`` passing its
  scalar operands first to the index maps and the kernel.
"""

from __future__ import annotations

import sys
import types

import numpy as np

WIDE = True  # float32 arithmetic of the reference is carried out in float64


class Arr(np.ndarray):
    """ndarray with jax's functional ``.at[idx].set(v)``."""

    @property
    def at(self):
        return _At(self)


class _At:
    def __init__(self, a):
        self._a = a

    def __getitem__(self, idx):
        a = self._a

        class _Upd:
            def set(self_inner, v):
                out = np.array(a, copy=True)
                out[idx] = v
                return out.view(Arr)
        return _Upd()


def _wrap(x):
    if isinstance(x, np.ndarray) and not isinstance(x, Arr):
        return x.view(Arr)
    return x


def _f32():
    return np.float64 if WIDE else np.float32


def _build_jnp():
    jnp = types.ModuleType("jax.numpy")

    def _fwd(name):
        fn = getattr(np, name)

        def call(*a, **kw):
            a = tuple(_f32() if x is _Float32 else x for x in a)
            if kw.get("dtype") is _Float32:
                kw["dtype"] = _f32()
            return _wrap(fn(*a, **kw))
        return call

    for name in ("zeros", "ones", "full", "full_like", "zeros_like", "ones_like", "where", "maximum",
                 "minimum", "exp", "log", "sum", "mean", "square", "concatenate", "arange", "outer",
                 "cos", "sin", "repeat", "einsum", "argmax", "max", "min", "logical_and", "logical_or",
                 "stack", "isfinite", "all", "abs", "sqrt", "tanh", "allclose", "array_equal"):
        setattr(jnp, name, _fwd(name))

    def asarray(x, dtype=None):
        if dtype is _Float32:
            dtype = _f32()
        return _wrap(np.asarray(x, dtype=dtype))

    def dot(a, b, preferred_element_type=None):
        return _wrap(np.dot(a, b))

    jnp.asarray = asarray
    jnp.array = asarray
    jnp.dot = dot
    jnp.float32 = _Float32
    jnp.float64 = np.float64
    jnp.int32 = np.int32
    jnp.bfloat16 = _Float32  # never reached by the generator's cases
    jnp.ndarray = np.ndarray
    return jnp


class _Float32Meta(type):
    """``jnp.float32``: a dtype-like whose numpy dtype follows ``WIDE``."""

    def __call__(cls, x):
        return _f32()(x)

    @property
    def dtype(cls):
        return np.dtype(_f32())


class _Float32(metaclass=_Float32Meta):
    pass


def _astype_patch():
    """``x.astype(jnp.float32)`` on an Arr: map the stand-in class to a dtype."""
    orig = np.ndarray.astype

    def astype(self, dtype, *a, **kw):
        if dtype is _Float32:
            dtype = _f32()
        return _wrap(orig(self, dtype, *a, **kw))
    Arr.astype = astype


def _build_lax():
    lax = types.ModuleType("jax.lax")

    def broadcasted_iota(dtype, shape, dimension):
        idx = np.arange(shape[dimension], dtype=np.int64)
        view = [1] * len(shape)
        view[dimension] = shape[dimension]
        return _wrap(np.broadcast_to(idx.reshape(view), shape).astype(np.int32))

    def rsqrt(x):
        return _wrap(1.0 / np.sqrt(x))

    def dynamic_update_slice(operand, update, start_indices):
        out = np.array(operand, copy=True)
        sl = []
        for dim, upd, s in zip(operand.shape, update.shape, start_indices):
            s = int(min(max(int(s), 0), dim - upd))  # jax clamps the start
            sl.append(slice(s, s + upd))
        out[tuple(sl)] = update
        return _wrap(out)

    def dynamic_update_slice_in_dim(operand, update, start_index, axis):
        starts = [0] * operand.ndim
        starts[axis] = start_index
        return dynamic_update_slice(operand, update, starts)

    lax.broadcasted_iota = broadcasted_iota
    lax.rsqrt = rsqrt
    lax.dynamic_update_slice = dynamic_update_slice
    lax.dynamic_update_slice_in_dim = dynamic_update_slice_in_dim
    return lax


def _build_nn():
    nn = types.ModuleType("jax.nn")

    def softmax(x, axis=-1):
        e = np.exp(x - np.max(x, axis=axis, keepdims=True))
        return _wrap(e / np.sum(e, axis=axis, keepdims=True))

    def silu(x):
        return _wrap(x / (1.0 + np.exp(-x)))

    nn.softmax = softmax
    nn.silu = silu
    return nn


def _build_random():
    """``jax.random`` with numpy streams, NOT jax's threefry: a key is a pair of
    uint32 words seeding ``numpy.random.default_rng``.  The values differ from
    jax's, which is why every golden file stores the inputs it was made from."""
    rnd = types.ModuleType("jax.random")

    def PRNGKey(seed):
        return np.array([0, int(seed) & 0xFFFFFFFF], dtype=np.uint32)

    def split(key, num=2):
        rng = np.random.default_rng([int(x) for x in np.asarray(key).ravel()])
        return rng.integers(0, 2**32, size=(num, 2), dtype=np.uint64).astype(np.uint32)

    def normal(key, shape=(), dtype=None):
        rng = np.random.default_rng([int(x) for x in np.asarray(key).ravel()])
        x = rng.standard_normal(shape).astype(np.float32)  # float32-representable draws
        return _wrap(x.astype(_f32()))

    rnd.PRNGKey, rnd.split, rnd.normal = PRNGKey, split, normal
    return rnd


class _CustomVjp:
    def __init__(self, fun, nondiff_argnums=()):
        self.fun = fun
        self.fwd = self.bwd = None

    def defvjp(self, fwd, bwd):
        self.fwd, self.bwd = fwd, bwd

    def __call__(self, *args):
        return self.fun(*args)


# --------------------------------------------------------------------------- #
# Pallas
# --------------------------------------------------------------------------- #
class _Grid:
    ids: tuple = ()
    dims: tuple = ()


class BlockSpec:
    def __init__(self, block_shape, index_map):
        self.block_shape = tuple(block_shape)
        self.index_map = index_map


class VMEM:
    def __init__(self, shape, dtype):
        self.shape = tuple(shape)
        self.dtype = _f32() if dtype is _Float32 else dtype


class CompilerParams:
    def __init__(self, **kw):
        self.kw = kw


class PrefetchScalarGridSpec:
    def __init__(self, num_scalar_prefetch, grid, in_specs, out_specs, scratch_shapes=()):
        self.num_scalar_prefetch = num_scalar_prefetch
        self.grid = tuple(grid)
        self.in_specs = in_specs
        self.out_specs = out_specs
        self.scratch_shapes = scratch_shapes


class ShapeDtypeStruct:
    def __init__(self, shape, dtype):
        self.shape = tuple(shape)
        self.dtype = _f32() if dtype is _Float32 else np.dtype(dtype)


def program_id(axis):
    return _Grid.ids[axis]


def num_programs(axis):
    return _Grid.dims[axis]


def when(cond):
    def deco(f):
        if bool(cond):
            f()
        return f
    return deco


def cdiv(a, b):
    return -(-a // b)


def _block_slices(spec, block_idx):
    return tuple(slice(i * b, (i + 1) * b) for i, b in zip(block_idx, spec.block_shape))


def _read_block(arr, spec, block_idx):
    sl = _block_slices(spec, block_idx)
    view = arr[sl]
    if view.shape == spec.block_shape:
        return _wrap(np.array(view, copy=True))
    pad = np.full(spec.block_shape, np.nan, dtype=arr.dtype)
    pad[tuple(slice(0, s) for s in view.shape)] = view
    return _wrap(pad)


def pallas_call(kernel, *, out_shape, grid=None, in_specs=None, out_specs=None, scratch_shapes=(),
                grid_spec=None, compiler_params=None, interpret=False, name=None, **_):
    n_scalar = 0
    if grid_spec is not None:
        n_scalar = grid_spec.num_scalar_prefetch
        grid, in_specs = grid_spec.grid, grid_spec.in_specs
        out_specs, scratch_shapes = grid_spec.out_specs, grid_spec.scratch_shapes
    single = not isinstance(out_shape, (list, tuple))
    out_shapes = [out_shape] if single else list(out_shape)
    o_specs = [out_specs] if isinstance(out_specs, BlockSpec) else list(out_specs)

    def run(*args):
        scalars = [np.asarray(a) for a in args[:n_scalar]]
        arrays = [np.asarray(a) for a in args[n_scalar:]]
        outs = [np.full(s.shape, np.nan, dtype=s.dtype) if np.issubdtype(s.dtype, np.floating)
                else np.zeros(s.shape, dtype=s.dtype) for s in out_shapes]
        scratch = [_wrap(np.zeros(s.shape, dtype=s.dtype)) for s in scratch_shapes]
        _Grid.dims = tuple(grid)
        for ids in np.ndindex(*grid):
            _Grid.ids = tuple(int(i) for i in ids)
            in_refs = [_read_block(a, sp, sp.index_map(*ids, *scalars)) for a, sp in zip(arrays, in_specs)]
            out_idx = [sp.index_map(*ids, *scalars) for sp in o_specs]
            out_refs = [_read_block(o, sp, bi) for o, sp, bi in zip(outs, o_specs, out_idx)]
            kernel(*scalars, *in_refs, *out_refs, *scratch)
            for o, sp, bi, ref in zip(outs, o_specs, out_idx, out_refs):
                sl = _block_slices(sp, bi)
                view = o[sl]
                view[...] = ref[tuple(slice(0, s) for s in view.shape)]
        res = [_wrap(o) for o in outs]
        return res[0] if single else res
    return run


def install(wide: bool = True) -> None:
    """Registers ``jax``, ``jax.numpy``, ``jax.lax``, ``jax.nn``, ``jax.random``
    and ``jax.experimental.pallas(.tpu)`` in ``sys.modules``."""
    global WIDE
    WIDE = wide
    _astype_patch()
    jax = types.ModuleType("jax")
    jnp, lax, nn = _build_jnp(), _build_lax(), _build_nn()
    rnd = _build_random()
    exp = types.ModuleType("jax.experimental")
    pl = types.ModuleType("jax.experimental.pallas")
    tpu = types.ModuleType("jax.experimental.pallas.tpu")
    for n in ("BlockSpec", "pallas_call", "program_id", "num_programs", "when", "cdiv"):
        setattr(pl, n, globals()[n])
    tpu.VMEM, tpu.CompilerParams, tpu.PrefetchScalarGridSpec = VMEM, CompilerParams, PrefetchScalarGridSpec
    pl.tpu = tpu
    exp.pallas = pl
    jax.numpy, jax.lax, jax.nn, jax.random, jax.experimental = jnp, lax, nn, rnd, exp
    jax.Array = np.ndarray
    jax.ShapeDtypeStruct = ShapeDtypeStruct
    jax.custom_vjp = _CustomVjp
    jax.jit = lambda f=None, **kw: f if f is not None else (lambda g: g)
    for mod_name, mod in (("jax", jax), ("jax.numpy", jnp), ("jax.lax", lax), ("jax.nn", nn),
                          ("jax.random", rnd), ("jax.experimental", exp),
                          ("jax.experimental.pallas", pl), ("jax.experimental.pallas.tpu", tpu)):
        sys.modules[mod_name] = mod
