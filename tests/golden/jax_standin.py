"""A minimal NumPy stand-in for the parts of jax / flax.nnx the reference's
retrieval path imports, so the reference's own Python functions can be
executed here (JAX is not installable in this environment).

Used only by make_golden.py to produce golden fixtures.  Each primitive
restates its published contract:

* jnp.*            -> numpy; jnp.dot keeps the input dtype (bf16 in -> bf16 out,
                      f32 in -> f32 out), accumulating in float32
* jax.lax.top_k    -> values descending along the last axis, lower index first
                      among equal values
* jax.lax.all_gather(x, axis, axis=0, tiled=False) -> stacks every device's x
* jax.lax.axis_index(axis) -> this device's position on the mesh axis
* shard_map        -> runs the body once per device in its own thread; inputs
                      with P(axis, None) are split by rows, P() replicated;
                      collectives rendezvous through a barrier
* flax.nnx         -> Module / Param / Variable / Rngs placeholders
"""
from __future__ import annotations

import functools
import sys
import threading
import types

import numpy as np

try:
    import ml_dtypes

    _BF16 = np.dtype(ml_dtypes.bfloat16)
except ImportError:  # pragma: no cover
    _BF16 = None


def _top_k(x, k):
    x = np.asarray(x)
    n = x.shape[-1]
    order = np.argsort(-x.astype(np.float64), axis=-1, kind="stable")[..., :k]
    return np.take_along_axis(x, order, axis=-1), order.astype(np.int32)


def _dot(a, b):
    a = np.asarray(a)
    b = np.asarray(b)
    out_dtype = np.result_type(a.dtype, b.dtype)
    r = np.asarray(a, np.float32) @ np.asarray(b, np.float32)
    return r.astype(out_dtype)


def _sigmoid(x):
    x = np.asarray(x)
    return (1.0 / (1.0 + np.exp(-x))).astype(x.dtype)


def _softmax(x, axis=-1):
    x = np.asarray(x)
    e = np.exp(x - np.max(x, axis=axis, keepdims=True))
    return e / np.sum(e, axis=axis, keepdims=True)


class _ShardCtx(threading.local):
    index = 0
    coll = None


_ctx = _ShardCtx()


class _Collective:
    def __init__(self, n):
        self.n = n
        self.barrier = threading.Barrier(n)
        self.slots = [None] * n

    def all_gather(self, x):
        i = _ctx.index
        self.slots[i] = np.asarray(x)
        self.barrier.wait()
        out = np.stack(self.slots, axis=0)
        self.barrier.wait()
        return out


def _all_gather(x, axis_name, axis=0, tiled=False):
    if axis != 0 or tiled:
        raise NotImplementedError("stand-in supports all_gather(axis=0, tiled=False)")
    return _ctx.coll.all_gather(x)


def _axis_index(axis_name):
    return np.int32(_ctx.index)


class PartitionSpec(tuple):
    def __new__(cls, *parts):
        return super().__new__(cls, parts)


class Mesh:
    def __init__(self, devices, axis_names):
        self.devices = np.asarray(devices)
        self.axis_names = tuple(axis_names)

    @property
    def size(self):
        return int(self.devices.size)


class NamedSharding:
    def __init__(self, mesh, spec):
        self.mesh, self.spec = mesh, spec


def shard_map(f, mesh, in_specs, out_specs, check_rep=True):
    n = mesh.size

    def run(*args):
        shards = []
        for a, spec in zip(args, in_specs):
            a = np.asarray(a)
            if len(spec) and spec[0] is not None:
                rows = a.shape[0] // n
                shards.append([a[i * rows:(i + 1) * rows] for i in range(n)])
            else:
                shards.append([a] * n)
        coll = _Collective(n)
        results = [None] * n
        errors = []

        def body(i):
            _ctx.index, _ctx.coll = i, coll
            try:
                results[i] = f(*[s[i] for s in shards])
            except Exception as e:  # pragma: no cover - surfaced below
                errors.append(e)
                coll.barrier.abort()

        threads = [threading.Thread(target=body, args=(i,)) for i in range(n)]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        if errors:
            raise errors[0]
        # out_specs P(): replicated results; every device must agree
        for r in results[1:]:
            for a, b in zip(r, results[0]):
                if not np.array_equal(a, b):
                    raise AssertionError("replicated shard_map outputs differ across devices")
        return results[0]

    return run


def jit(fun=None, *, static_argnames=(), **_):
    if fun is None:
        return lambda f: f
    return fun


class _Var:
    def __init__(self, value=None, **_):
        self.value = value


class Module:
    pass


class LayerNorm:
    """flax.nnx.LayerNorm's published computation over the last axis (epsilon 1e-6,
    fast variance): mean, var = max(mean(x^2) - mean^2, 0),
    (x - mean) / sqrt(var + eps) * scale + bias, in float32."""

    def __init__(self, num_features, *, epsilon=1e-6, rngs=None, scale=None, bias=None):
        self.epsilon = epsilon
        self.scale = _Var(np.ones(num_features, np.float32) if scale is None else scale)
        self.bias = _Var(np.zeros(num_features, np.float32) if bias is None else bias)

    def __call__(self, x):
        x = np.asarray(x, np.float32)
        mean = x.mean(axis=-1, keepdims=True)
        var = np.maximum((x * x).mean(axis=-1, keepdims=True) - mean * mean, 0.0)
        y = (x - mean) / np.sqrt(var + np.float32(self.epsilon))
        return (y * self.scale.value + self.bias.value).astype(np.float32)


class Rngs:
    def __init__(self, *a, **k):
        pass


def install() -> None:
    """Register the stand-in modules in sys.modules (jax, jax.numpy, ..., flax.nnx)."""
    jax = types.ModuleType("jax")
    jnp = types.ModuleType("jax.numpy")
    for name in ("einsum", "exp", "sum", "arange", "zeros", "ones", "full", "asarray", "array",
                 "concatenate", "where", "tril", "broadcast_to", "outer", "sqrt", "mean",
                 "float32", "int32"):
        setattr(jnp, name, getattr(np, name))
    jnp.bfloat16 = _BF16
    jnp.dot = _dot
    jnp.linalg = np.linalg
    lax = types.ModuleType("jax.lax")
    lax.top_k = _top_k
    lax.all_gather = _all_gather
    lax.axis_index = _axis_index
    nn = types.ModuleType("jax.nn")
    nn.sigmoid = _sigmoid
    nn.softmax = _softmax
    experimental = types.ModuleType("jax.experimental")
    pallas = types.ModuleType("jax.experimental.pallas")

    def _no_pallas(*a, **k):
        raise NotImplementedError("Pallas kernels do not run in the stand-in")

    pallas.pallas_call = _no_pallas
    pallas.BlockSpec = _no_pallas
    pallas.no_block_spec = None
    sm = types.ModuleType("jax.experimental.shard_map")
    sm.shard_map = shard_map
    experimental.pallas = pallas
    experimental.shard_map = sm
    sharding = types.ModuleType("jax.sharding")
    sharding.PartitionSpec = PartitionSpec
    sharding.NamedSharding = NamedSharding
    sharding.Mesh = Mesh
    jax.numpy, jax.lax, jax.nn = jnp, lax, nn
    jax.experimental, jax.sharding = experimental, sharding
    jax.jit = jit
    jax.Array = np.ndarray
    flax = types.ModuleType("flax")
    nnx = types.ModuleType("flax.nnx")
    nnx.Module, nnx.Param, nnx.Variable, nnx.Rngs = Module, _Var, _Var, Rngs
    nnx.LayerNorm = LayerNorm
    flax.nnx = nnx
    sys.modules.update({
        "jax": jax, "jax.numpy": jnp, "jax.lax": lax, "jax.nn": nn,
        "jax.experimental": experimental, "jax.experimental.pallas": pallas,
        "jax.experimental.shard_map": sm, "jax.sharding": sharding,
        "flax": flax, "flax.nnx": nnx,
    })
