"""NumPy-backed stand-in for the subset of ``mlx.core`` that TurboPolar's CPU path uses.

Test infrastructure only: ``tests/golden/make_golden.py`` puts this package first on
``sys.path`` so that the reference's own Python sources (encoder, decoder, V quantizer,
cache runtime, storage, the Metal bridge's CPU fallback and the Llama adapter) execute
unmodified on this machine, where MLX cannot be installed.  Nothing in the product imports
this module.

Numerics model (what "MLX on CPU" is taken to compute; MLX's own CPU kernels are not
available to measure against):

* Binary operators follow MLX's promotion rules, which coincide with NumPy NEP 50: a Python
  scalar is weakly typed and takes the array's dtype (``float16_array + np.pi`` stays
  float16 with pi rounded to 3.140625); two arrays promote (float16 with float32 gives
  float32).  ``mx.array(0.0)`` is a strongly typed float32 scalar.
* float16 ``+ - * /`` round once to float16 (NumPy evaluates them in float32 and rounds,
  which is the correctly rounded float16 result).
* ``sqrt, log, exp, sin, cos, arctan2`` are evaluated in float64, rounded to float32 and
  then to the array dtype: a correctly rounded float32 libm, then the float16 store.
* ``round`` is half-to-even.  float16 sums accumulate in float32.  ``softmax`` of a
  float16 array is evaluated in float32 and rounded back.
"""

from __future__ import annotations

import numpy as np

__all__ = ["array"]


class Dtype:
    def __init__(self, np_dtype, name):
        self.np = np.dtype(np_dtype)
        self.name = name

    @property
    def size(self):
        return self.np.itemsize

    def __eq__(self, other):
        return isinstance(other, Dtype) and self.np == other.np

    def __hash__(self):
        return hash(self.np)

    def __repr__(self):
        return f"mlx.core.{self.name}"


float16 = Dtype(np.float16, "float16")
float32 = Dtype(np.float32, "float32")
float64 = Dtype(np.float64, "float64")
int8 = Dtype(np.int8, "int8")
int16 = Dtype(np.int16, "int16")
int32 = Dtype(np.int32, "int32")
int64 = Dtype(np.int64, "int64")
uint8 = Dtype(np.uint8, "uint8")
uint16 = Dtype(np.uint16, "uint16")
uint32 = Dtype(np.uint32, "uint32")
bool_ = Dtype(np.bool_, "bool_")
_ALL = [float16, float32, float64, int8, int16, int32, int64, uint8, uint16, uint32, bool_]
_BY_NP = {d.np: d for d in _ALL}


def _to_np_dtype(dtype):
    if dtype is None:
        return None
    if isinstance(dtype, Dtype):
        return dtype.np
    return np.dtype(dtype)


def _raw(x):
    """Unwrap an operand: arrays to ndarrays, Python scalars stay weak."""
    if isinstance(x, array):
        return x._a
    return x


class array:
    __array_priority__ = 1000

    def __init__(self, value, dtype=None):
        npd = _to_np_dtype(dtype)
        if isinstance(value, array):
            a = value._a
        elif isinstance(value, np.ndarray):
            a = value
        elif isinstance(value, bool):
            a = np.array(value, dtype=np.bool_)
        elif isinstance(value, int):
            a = np.array(value, dtype=np.int32)
        elif isinstance(value, float):
            a = np.array(value, dtype=np.float32)
        else:
            a = np.array(value)
            if a.dtype == np.float64:
                a = a.astype(np.float32)
            elif a.dtype == np.int64:
                a = a.astype(np.int32)
        if npd is not None:
            a = a.astype(npd)
        self._a = np.array(a, copy=True) if a.base is not None and isinstance(value, np.ndarray) else a

    @classmethod
    def _wrap(cls, a):
        obj = cls.__new__(cls)
        obj._a = np.asarray(a)
        return obj

    # ------------------------------------------------------------------ attributes
    @property
    def shape(self):
        return tuple(int(s) for s in self._a.shape)

    @property
    def ndim(self):
        return self._a.ndim

    @property
    def size(self):
        return int(self._a.size)

    @property
    def itemsize(self):
        return int(self._a.itemsize)

    @property
    def nbytes(self):
        return int(self._a.nbytes)

    @property
    def dtype(self):
        return _BY_NP[self._a.dtype]

    def __array__(self, dtype=None, copy=None):
        return self._a if dtype is None else self._a.astype(dtype)

    def __len__(self):
        return len(self._a)

    def __repr__(self):
        return f"array({self._a!r})"

    def item(self):
        return self._a.item()

    def tolist(self):
        return self._a.tolist()

    # ------------------------------------------------------------------ shape ops
    def reshape(self, *shape):
        if len(shape) == 1 and isinstance(shape[0], (tuple, list)):
            shape = tuple(shape[0])
        return array._wrap(self._a.reshape(shape))

    def astype(self, dtype):
        return array._wrap(self._a.astype(_to_np_dtype(dtype)))

    def transpose(self, *axes):
        if len(axes) == 1 and isinstance(axes[0], (tuple, list)):
            axes = tuple(axes[0])
        return array._wrap(np.transpose(self._a, axes or None))

    def squeeze(self, axis=None):
        return array._wrap(np.squeeze(self._a, axis=axis))

    def sum(self, axis=None, keepdims=False):
        return sum(self, axis=axis, keepdims=keepdims)

    def max(self, axis=None, keepdims=False):
        return max(self, axis=axis, keepdims=keepdims)

    def all(self, axis=None, keepdims=False):
        return all(self, axis=axis, keepdims=keepdims)

    def __getitem__(self, idx):
        if isinstance(idx, array):
            idx = idx._a
        elif isinstance(idx, tuple):
            idx = tuple(i._a if isinstance(i, array) else i for i in idx)
        return array._wrap(self._a[idx])

    def __setitem__(self, idx, value):
        if isinstance(idx, tuple):
            idx = tuple(i._a if isinstance(i, array) else i for i in idx)
        self._a[idx] = _raw(value)

    # ------------------------------------------------------------------ operators
    def _bin(self, other, op, reverse=False):
        a, b = self._a, _raw(other)
        return array._wrap(op(b, a) if reverse else op(a, b))

    def __add__(self, o): return self._bin(o, np.add)
    def __radd__(self, o): return self._bin(o, np.add, True)
    def __sub__(self, o): return self._bin(o, np.subtract)
    def __rsub__(self, o): return self._bin(o, np.subtract, True)
    def __mul__(self, o): return self._bin(o, np.multiply)
    def __rmul__(self, o): return self._bin(o, np.multiply, True)
    def __truediv__(self, o): return self._bin(o, _true_divide)
    def __rtruediv__(self, o): return self._bin(o, _true_divide, True)
    def __pow__(self, o): return self._bin(o, np.power)
    def __and__(self, o): return self._bin(o, np.bitwise_and)
    def __rand__(self, o): return self._bin(o, np.bitwise_and, True)
    def __or__(self, o): return self._bin(o, np.bitwise_or)
    def __ror__(self, o): return self._bin(o, np.bitwise_or, True)
    def __xor__(self, o): return self._bin(o, np.bitwise_xor)
    def __lshift__(self, o): return self._bin(o, np.left_shift)
    def __rshift__(self, o): return self._bin(o, np.right_shift)
    def __lt__(self, o): return self._bin(o, np.less)
    def __le__(self, o): return self._bin(o, np.less_equal)
    def __gt__(self, o): return self._bin(o, np.greater)
    def __ge__(self, o): return self._bin(o, np.greater_equal)
    def __eq__(self, o): return self._bin(o, np.equal)
    def __ne__(self, o): return self._bin(o, np.not_equal)
    def __neg__(self): return array._wrap(-self._a)
    def __abs__(self): return array._wrap(np.abs(self._a))
    def __invert__(self): return array._wrap(~self._a)
    __hash__ = None

    def __matmul__(self, o):
        return matmul(self, o)

    def __bool__(self):
        return bool(self._a)

    def __float__(self):
        return float(self._a)

    def __int__(self):
        return int(self._a)


def _true_divide(a, b):
    out = np.true_divide(a, b)
    # Integer / integer in MLX yields float32 (NumPy gives float64).
    if out.dtype == np.float64 and not (
        (isinstance(a, np.ndarray) and a.dtype == np.float64)
        or (isinstance(b, np.ndarray) and b.dtype == np.float64)
    ):
        out = out.astype(np.float32)
    return out


# ---------------------------------------------------------------------- elementwise
def _transcendental(fn, *xs):
    arrs = [np.asarray(_raw(x)) for x in xs]
    dt = np.result_type(*arrs)
    if not np.issubdtype(dt, np.floating):
        dt = np.dtype(np.float32)
    r64 = fn(*[a.astype(np.float64) for a in arrs])
    return array._wrap(r64.astype(np.float32).astype(dt))


def sqrt(x): return _transcendental(np.sqrt, x)
def log(x): return _transcendental(np.log, x)
def exp(x): return _transcendental(np.exp, x)
def cos(x): return _transcendental(np.cos, x)
def sin(x): return _transcendental(np.sin, x)
def arctan2(a, b): return _transcendental(np.arctan2, a, b)


def abs(x): return array._wrap(np.abs(_raw(x)))
def maximum(a, b): return array._wrap(np.maximum(_raw(a), _raw(b)))
def minimum(a, b): return array._wrap(np.minimum(_raw(a), _raw(b)))
def round(x, decimals=0): return array._wrap(np.round(_raw(x), decimals))
def clip(x, a_min, a_max): return array._wrap(np.clip(_raw(x), _raw(a_min), _raw(a_max)))
def isfinite(x): return array._wrap(np.isfinite(_raw(x)))
def where(c, x, y): return array._wrap(np.where(_raw(c), _raw(x), _raw(y)))
def contiguous(x): return array._wrap(np.ascontiguousarray(_raw(x)))
def equal(a, b): return array._wrap(np.equal(_raw(a), _raw(b)))


# ---------------------------------------------------------------------- reductions
def _axis(axis):
    return tuple(axis) if isinstance(axis, list) else axis


def sum(x, axis=None, keepdims=False):
    a = _raw(x)
    if a.dtype == np.float16:
        return array._wrap(np.sum(a.astype(np.float32), axis=_axis(axis), keepdims=keepdims).astype(np.float16))
    if a.dtype == np.bool_ or np.issubdtype(a.dtype, np.integer):
        return array._wrap(np.sum(a, axis=_axis(axis), keepdims=keepdims).astype(a.dtype if a.dtype != np.bool_ else np.int32))
    return array._wrap(np.sum(a, axis=_axis(axis), keepdims=keepdims))


def max(x, axis=None, keepdims=False):
    return array._wrap(np.max(_raw(x), axis=_axis(axis), keepdims=keepdims))


def min(x, axis=None, keepdims=False):
    return array._wrap(np.min(_raw(x), axis=_axis(axis), keepdims=keepdims))


def mean(x, axis=None, keepdims=False):
    a = _raw(x)
    r = np.mean(a.astype(np.float32), axis=_axis(axis), keepdims=keepdims)
    return array._wrap(r.astype(a.dtype if np.issubdtype(a.dtype, np.floating) else np.float32))


def all(x, axis=None, keepdims=False):
    return array._wrap(np.all(_raw(x), axis=_axis(axis), keepdims=keepdims))


def any(x, axis=None, keepdims=False):
    return array._wrap(np.any(_raw(x), axis=_axis(axis), keepdims=keepdims))


def softmax(x, axis=-1, precise=False):
    a = _raw(x)
    a32 = a.astype(np.float32)
    m = np.max(a32, axis=axis, keepdims=True)
    e = np.exp((a32 - m).astype(np.float64)).astype(np.float32)
    r = e / np.sum(e, axis=axis, keepdims=True)
    return array._wrap(r.astype(a.dtype))


def matmul(a, b):
    ra, rb = _raw(a), _raw(b)
    if ra.dtype == np.float16 and rb.dtype == np.float16:
        return array._wrap((ra.astype(np.float32) @ rb.astype(np.float32)).astype(np.float16))
    return array._wrap(np.matmul(ra, rb))


# ---------------------------------------------------------------------- construction
def zeros(shape, dtype=float32):
    return array._wrap(np.zeros(shape, dtype=_to_np_dtype(dtype)))


def ones(shape, dtype=float32):
    return array._wrap(np.ones(shape, dtype=_to_np_dtype(dtype)))


def full(shape, vals, dtype=None):
    v = _raw(vals)
    npd = _to_np_dtype(dtype)
    if npd is None:
        npd = np.asarray(v).dtype if isinstance(v, np.ndarray) else (np.float32 if isinstance(v, float) else np.int32)
    return array._wrap(np.full(shape, v, dtype=npd))


def arange(*args, dtype=None):
    a = np.arange(*args)
    if a.dtype == np.int64:
        a = a.astype(np.int32)
    elif a.dtype == np.float64:
        a = a.astype(np.float32)
    if dtype is not None:
        a = a.astype(_to_np_dtype(dtype))
    return array._wrap(a)


def tril(x, k=0):
    return array._wrap(np.tril(_raw(x), k))


def concatenate(xs, axis=0):
    return array._wrap(np.concatenate([_raw(x) for x in xs], axis=axis))


def stack(xs, axis=0):
    return array._wrap(np.stack([_raw(x) for x in xs], axis=axis))


def expand_dims(x, axis):
    return array._wrap(np.expand_dims(_raw(x), axis))


def squeeze(x, axis=None):
    return array._wrap(np.squeeze(_raw(x), axis=axis))


def repeat(x, repeats, axis=None):
    return array._wrap(np.repeat(_raw(x), repeats, axis=axis))


def pad(x, pad_width, constant_values=0):
    return array._wrap(np.pad(_raw(x), pad_width, constant_values=constant_values))


def eval(*args):
    return None


class _Metal:
    @staticmethod
    def is_available():
        return False


metal = _Metal()


class _Fast:
    """``mx.fast.metal_kernel`` builds an object whose dispatch raises: the reference's
    dispatch probe (``rfsn_v11/kernels/turbo_polar/metal.py:13-54``) then reports the
    Metal path unsupported and every bridge call takes its CPU fallback."""

    @staticmethod
    def metal_kernel(name, input_names, output_names, source, header="", **kw):
        def _dispatch(*a, **k):
            raise RuntimeError(f"Metal kernel {name} cannot run here")
        return _dispatch


fast = _Fast()


class _Random:
    def __init__(self):
        self._rng = np.random.default_rng(0)

    def seed(self, s):
        self._rng = np.random.default_rng(s)

    def normal(self, shape=(), dtype=float32, loc=0.0, scale=1.0):
        a = self._rng.standard_normal(tuple(shape)).astype(np.float32) * scale + loc
        return array._wrap(a.astype(_to_np_dtype(dtype)))


random = _Random()
