"""Pure-Python stand-in for the part of NVIDIA Warp that gswarp's kernel
modules use, so that the reference's own kernel bodies can run on the CPU
where ``warp-lang`` is not installed.

TEST INFRASTRUCTURE ONLY.  ``make_kernel_golden.py`` loads gswarp's kernel
modules through ``load_module`` (which installs this module as ``warp``) and
runs their ``@wp.kernel`` bodies with ``launch`` to produce golden vectors.
Nothing in the product imports it.

Semantics (those of a Warp kernel compiled without fast math and without
contraction, evaluated in the source's order):

* Every float literal of a loaded module is made binary32 before the module
  runs (Warp compiles literals as float32), and ``a / b`` of two integers is
  an integer division (Warp's ``/`` on ints); float scalars are numpy
  ``float32``, so each operation rounds once, in the source's evaluation
  order, with no fused multiply-add.  ``float()`` inside a kernel is
  ``float32``.
* ``vec2/3/4`` are float32 numpy arrays with elementwise arithmetic;
  ``vec2i/vec4i`` are int tuples.
* ``exp``: the C library's ``expf``; ``log``: the logarithm evaluated in
  double and rounded to binary32 (the correctly rounded binary32 log);
  ``sqrt``: the correctly rounded binary32 square root.  Float-to-int
  conversions truncate toward zero and saturate (NaN -> 0).
* A kernel that uses tile collectives becomes a generator (the loader turns
  every ``wp.tile(x)`` into a ``yield``); ``launch`` steps the threads of a
  block in lockstep from one ``tile`` to the next and hands each the block's
  values, like the barrier of a real block.  ``tile_load`` copies memory an
  earlier launch wrote, so it needs no exchange.
  ``tile_sum`` / ``tile_reduce(add)`` of floats accumulate in float64 and
  ``atomic_add`` / ``tile_atomic_add`` add into float64 arrays: the
  reference's own order (a warp shuffle tree, unordered atomics) is not
  fixed, so the golden value is the exact sum of the float32 terms.
"""

from __future__ import annotations

import ast
import ctypes
import ctypes.util
import math
import sys
import types
from pathlib import Path

import numpy as np

F32 = np.float32

_libm = ctypes.CDLL(ctypes.util.find_library("m") or "libm.so.6")
_libm.expf.restype = ctypes.c_float
_libm.expf.argtypes = [ctypes.c_float]


# ---------------------------------------------------------------- scalar types
def float32(x=0.0):
    return F32(x)


def _sat_int(x, lo, hi):
    if isinstance(x, (float, np.floating)):
        if math.isnan(float(x)):
            return 0
        v = math.trunc(float(x)) if math.isfinite(float(x)) else (hi if x > 0 else lo)
        return int(min(max(v, lo), hi))
    return int(x)


def int32(x=0):
    v = _sat_int(x, -(1 << 31), (1 << 31) - 1)
    return int(np.int64(v).astype(np.int32))


def uint32(x=0):
    if isinstance(x, (float, np.floating)):
        return np.uint32(_sat_int(x, 0, (1 << 32) - 1))
    return np.uint32(int(x) & 0xFFFFFFFF)


def int64(x=0):
    return np.int64(int(x))


def uint64(x=0):
    return np.uint64(int(x) & 0xFFFFFFFFFFFFFFFF)


float16 = float32
bool_ = bool


def vec2(*a):
    return np.array(a if a else (0.0, 0.0), dtype=F32)


def vec3(*a):
    return np.array(a if a else (0.0, 0.0, 0.0), dtype=F32)


def vec4(*a):
    return np.array(a if a else (0.0, 0.0, 0.0, 0.0), dtype=F32)


def vec2i(*a):
    return tuple(int(v) for v in a)


def vec4i(*a):
    return tuple(int(v) for v in a)


# ------------------------------------------------------------------- builtins
def exp(x):
    return F32(_libm.expf(float(x)))


def log(x):
    return F32(math.log(float(x)))


def sqrt(x):
    return np.sqrt(F32(x))


def floor(x):
    return np.floor(F32(x))


def ceil(x):
    return np.ceil(F32(x))


def abs(x):  # noqa: A001 - Warp's name
    return np.abs(x)


def min(a, b):  # noqa: A001
    return a if a < b else b


def max(a, b):  # noqa: A001
    return a if a > b else b


def clamp(x, lo, hi):
    return min(max(x, lo), hi)


def dot(a, b):
    s = a[0] * b[0]
    for i in range(1, len(a)):
        s = s + a[i] * b[i]
    return s


def add(a, b):
    return a + b


def cast(x, dtype):
    if dtype is int32:
        return int(F32(x).view(np.int32))
    raise NotImplementedError(f"cast to {dtype}")


def constant(x):
    return x


def init():  # module-level call of the loaded modules; nothing to set up
    return None


def array(*_a, **_k):  # type annotations only
    return None


array2d = array3d = array


# ------------------------------------------------------------------- arrays
class WArray:
    """A Warp array over a numpy buffer.  ``vec`` > 0: elements are float32
    vectors of that length (reads return copies).  A float64 buffer is the
    target of atomic adds."""

    def __init__(self, data: np.ndarray, vec: int = 0):
        self.data = data
        self.vec = vec

    @property
    def shape(self):
        return self.data.shape[:-1] if self.vec else self.data.shape

    def __len__(self):
        return self.shape[0]

    def __getitem__(self, i):
        v = self.data[i]
        if self.vec:
            return v.astype(F32) if v.dtype != F32 else v.copy()
        if isinstance(v, np.integer):
            return int(v) if v.dtype != np.uint32 else v
        return v

    def __setitem__(self, i, v):
        self.data[i] = v


def warray(a, vec: int = 0) -> WArray:
    return WArray(a, vec)


# ----------------------------------------------------------- thread context
class _Ctx:
    tid = 0
    lane = 0



_ctx = _Ctx()


def tid():
    return _ctx.tid


class Tile:
    def __init__(self, values):
        self.values = values

    def __getitem__(self, idx):  # tile_load results: [0, row, col]
        return self.values[idx]


def tile(x, preserve_type=False):
    raise RuntimeError("wp.tile outside a loaded @wp.kernel body (the loader turns it into a yield)")


def _fsum(vals):
    if isinstance(vals[0], np.ndarray):
        return np.sum(np.stack([v.astype(np.float64) for v in vals]), axis=0)
    if isinstance(vals[0], (float, np.floating)):
        return math.fsum(float(v) for v in vals)
    return sum(int(v) for v in vals)


def tile_sum(t):
    return Tile([_fsum(t.values)])


def tile_reduce(op, t):
    if op is add:
        return Tile([_fsum(t.values)])
    if op is max or op is min:
        r = t.values[0]
        for v in t.values[1:]:
            r = op(r, v)
        return Tile([r])
    raise NotImplementedError(op)


def tile_extract(t, i):
    return t.values[i]


def atomic_add(arr: WArray, i, value):
    arr.data[i] = arr.data[i] + value


def atomic_min(arr: WArray, i, value):
    if value < arr.data[i]:
        arr.data[i] = value


def atomic_max(arr: WArray, i, value):
    if value > arr.data[i]:
        arr.data[i] = value


def tile_atomic_add(arr: WArray, t, offset=0):
    # a collective: every thread of the block calls it with the same tile;
    # the block adds it once
    if _ctx.lane == 0:
        arr.data[offset] = arr.data[offset] + np.asarray(t.values[0], dtype=np.float64)


def tile_load(arr: WArray, shape, offset, storage="shared"):
    """Tile of ``shape`` at ``offset`` (zero outside the array).  The source
    array was written by an earlier launch, so every thread reads the same
    values without an exchange."""
    src = arr.data
    out = np.zeros(shape, dtype=src.dtype)
    sl_src, sl_dst = [], []
    for o, s, n in zip(offset, shape, src.shape):
        a, b = builtins_max(o, 0), builtins_min(o + s, n)
        sl_src.append(slice(a, b))
        sl_dst.append(slice(a - o, b - o) if b > a else slice(0, 0))
    out[tuple(sl_dst)] = src[tuple(sl_src)]
    return Tile(out)


import builtins as _builtins  # noqa: E402

builtins_max = _builtins.max
builtins_min = _builtins.min


# ------------------------------------------------------------ kernel objects
class Kernel:
    def __init__(self, func):
        self.func = func
        self.key = func.__name__
        # a kernel with tile collectives was turned into a generator by the
        # loader; tile_load (a copy of memory an earlier launch wrote) needs
        # no exchange
        self.uses_tiles = bool(func.__code__.co_flags & 0x20)  # CO_GENERATOR


def kernel(func=None, **_kw):
    if func is None:
        return lambda f: Kernel(f)
    return Kernel(func)


def func(f=None, **_kw):
    if f is None:
        return lambda g: g
    return f


def launch(k: Kernel, dim: int, inputs, block_dim: int = 256):
    """Runs ``k`` over ``dim`` threads.  Kernels without tile collectives run
    thread by thread.  A kernel with them is a generator that yields at every
    ``tile``: the threads of a block are stepped in lockstep, each one up to
    its next ``tile``, and then every thread receives the block's values."""
    f = k.func
    if not k.uses_tiles:
        _ctx.block = None
        for t in range(dim):
            _ctx.tid = t
            f(*inputs)
        return
    for b0 in range(0, dim, block_dim):
        n = builtins_min(block_dim, dim - b0)
        gens = []
        for lane in range(n):
            _ctx.tid, _ctx.lane = b0 + lane, lane
            gens.append(f(*inputs))
        send = [None] * n
        alive = list(range(n))
        while alive:
            got = {}
            for lane in alive:
                _ctx.tid, _ctx.lane = b0 + lane, lane
                try:
                    v = gens[lane].send(send[lane])
                except StopIteration:
                    continue
                got[lane] = v.copy() if isinstance(v, np.ndarray) else v
            if got and len(got) != len(alive):
                raise RuntimeError(f"{k.key}: threads of a block diverged at a tile collective")
            if got:
                values = [got[lane] for lane in range(n)]
                for lane in got:
                    send[lane] = Tile(values)
            alive = list(got)


# ----------------------------------------------------------- module loading
class _F32Literals(ast.NodeTransformer):
    """float literal -> float32; ``a / b`` -> Warp division; inside a
    ``@wp.kernel`` body, ``wp.tile(x)`` -> ``(yield x)`` (the kernel becomes
    a generator that ``launch`` steps in lockstep with the block's other
    threads)."""

    def __init__(self):
        self.in_kernel = 0

    def visit_FunctionDef(self, node):
        is_kernel = any(isinstance(d, ast.Attribute) and d.attr == "kernel" for d in node.decorator_list)
        self.in_kernel += is_kernel
        self.generic_visit(node)
        self.in_kernel -= is_kernel
        return node

    def visit_Call(self, node):
        self.generic_visit(node)
        f = node.func
        if (self.in_kernel and isinstance(f, ast.Attribute) and f.attr == "tile"
                and isinstance(f.value, ast.Name) and f.value.id == "wp"):
            return ast.copy_location(ast.Yield(value=node.args[0]), node)
        return node

    def visit_Constant(self, node):
        if isinstance(node.value, float):
            return ast.copy_location(
                ast.Call(func=ast.Name("__wp_f32__", ast.Load()), args=[node], keywords=[]), node)
        return node

    def visit_BinOp(self, node):
        self.generic_visit(node)
        if isinstance(node.op, ast.Div):
            return ast.copy_location(
                ast.Call(func=ast.Name("__wp_div__", ast.Load()), args=[node.left, node.right], keywords=[]), node)
        return node


def _wp_div(a, b):
    ints = (int, np.integer)
    if isinstance(a, ints) and isinstance(b, ints) and not isinstance(a, bool):
        q = _builtins.abs(int(a)) // _builtins.abs(int(b))
        return q if (a >= 0) == (b >= 0) else -q
    return a / b


class _AnyModule(types.ModuleType):
    """Stub for host-only modules a kernel module imports names from."""

    def __getattr__(self, name):
        if name.startswith("__"):
            raise AttributeError(name)
        return lambda *a, **k: None


def _package(name: str, path: Path | None = None):
    if name not in sys.modules:
        m = types.ModuleType(name)
        m.__path__ = [str(path)] if path else []
        sys.modules[name] = m
    return sys.modules[name]


def install() -> types.ModuleType:
    """Makes ``import warp`` return this module."""
    me = sys.modules[__name__]
    sys.modules["warp"] = me
    return me


def stub(name: str) -> None:
    sys.modules[name] = _AnyModule(name)


def load_module(fullname: str, path: Path) -> types.ModuleType:
    """Loads one reference source file as module ``fullname`` (its package
    must exist in ``sys.modules``) with the literal/division transform."""
    install()
    tree = _F32Literals().visit(ast.parse(path.read_text(encoding="utf-8"), filename=str(path)))
    ast.fix_missing_locations(tree)
    mod = types.ModuleType(fullname)
    mod.__file__ = str(path)
    mod.__package__ = fullname.rpartition(".")[0]
    mod.__dict__.update(__wp_f32__=F32, __wp_div__=_wp_div, float=float32)
    sys.modules[fullname] = mod
    exec(compile(tree, str(path), "exec"), mod.__dict__)
    return mod


def package(name: str, path: Path | None = None):
    return _package(name, path)
