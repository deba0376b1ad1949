"""Host-side logic that needs no GPU: dtype resolution, broadcasting,
layout collapse and operand classification of the fusion planner,
reduction result dtypes, config."""

import numpy as np
import pytest

from macmetalpy_b200 import _broadcasting as bc
from macmetalpy_b200 import _fusion as fu
from macmetalpy_b200._config import get_config, set_config
from macmetalpy_b200._dtypes import resolve_dtype
from macmetalpy_b200.ndarray import _resolve
from macmetalpy_b200.reductions import out_dtype, scan_out_dtype


class FakeArray:
    def __init__(self, shape, dtype, strides=None, ptr=1 << 20):
        self._shape = tuple(shape)
        self._dtype = np.dtype(dtype)
        self._strides = tuple(strides) if strides is not None else fu._c_strides(self._shape)
        self._ptr = ptr
        self._fusion_node = None


def test_broadcast_shapes_rules():
    assert bc.broadcast_shapes((8192, 1), (1, 32768)) == (8192, 32768)
    assert bc.broadcast_shapes((2, 1, 3), (3, 1)) == (2, 3, 3)
    assert bc.broadcast_shapes((), (4,)) == (4,)
    with pytest.raises(ValueError):
        bc.broadcast_shapes((2, 3), (4,))
    assert bc.broadcast_strides((3, 1), (2, 3, 5), (1, 1)) == (0, 1, 0)


def test_resolve_dtype_matches_reference_rules():
    assert resolve_dtype(np.int8) == np.int16
    assert resolve_dtype(np.uint8) == np.uint16
    assert resolve_dtype(None) == np.float32
    assert resolve_dtype(np.float64) == np.float64  # cpu_fallback default: kept
    set_config(float64_behavior="downcast", warn_on_downcast=False)
    assert resolve_dtype(np.float64) == np.float32
    with pytest.raises(ValueError):
        set_config(float64_behavior="bogus")


def test_elementwise_dtype_resolution():
    f32, i32 = np.dtype(np.float32), np.dtype(np.int32)
    assert _resolve("add_op", (f32, float)) == (f32, f32)
    assert _resolve("add_op", (i32, float))[1] == np.float64
    assert _resolve("sqrt_op", (i32,))[1] == np.float64
    assert _resolve("floor_divide_op", (i32, i32)) == (i32, i32)
    assert _resolve("lt_op", (i32, f32)) == (np.float64, np.bool_)
    with pytest.raises(TypeError):
        _resolve("neg_op", (np.dtype(bool),))


def test_reduction_dtypes():
    assert out_dtype("sum", np.int32) == np.int64
    assert out_dtype("sum", np.uint16) == np.uint64
    assert out_dtype("sum", np.bool_) == np.int64
    assert out_dtype("mean", np.int32) == np.float64
    assert out_dtype("var", np.float16) == np.float16
    assert out_dtype("argmax", np.float32) == np.int64
    assert scan_out_dtype(np.int32) == np.int64
    assert scan_out_dtype(np.float32) == np.float32


def test_collapse_and_kinds():
    a = fu.InputNode(FakeArray((8192, 1), np.float32))
    b = fu.InputNode(FakeArray((1, 32768), np.float32))
    node = fu.BinaryOpNode("add_op", a, b, (8192, 32768), np.float32)
    p = fu._Plan(node, (8192, 32768), 4)
    assert p.cshape == [8192, 32768]
    assert p.kinds == ["sb", "sv"]
    assert p.vec_ok and not p.idx64
    # same-shape contiguous inputs collapse to one dimension
    c = fu.InputNode(FakeArray((64, 32, 16), np.float32))
    d = fu.InputNode(FakeArray((64, 32, 16), np.float32, ptr=(1 << 20) + 4096))
    p2 = fu._Plan(fu.BinaryOpNode("mul_op", c, d, (64, 32, 16), np.float32), (64, 32, 16), 4)
    assert p2.kinds == ["ct", "ct"] and not p2.strided
    # misaligned contiguous input disables the vector path
    e = fu.InputNode(FakeArray((100,), np.float32, ptr=(1 << 20) + 4))
    p3 = fu._Plan(fu.UnaryOpNode("exp_op", e, (100,), np.float32), (100,), 4)
    assert p3.kinds == ["ctu"] and not p3.vec_ok
    # transposed view is a general gather
    t = fu.InputNode(FakeArray((32, 64), np.float32, strides=(1, 32)))
    p4 = fu._Plan(fu.UnaryOpNode("exp_op", t, (32, 64), np.float32), (32, 64), 4)
    assert p4.kinds == ["sg"] and p4.cstrides == [[1, 32]]
    # more than 2^31 elements switches to 64-bit indexing
    big = fu.InputNode(FakeArray((1 << 16, 1), np.float32))
    big2 = fu.InputNode(FakeArray((1, 1 << 16), np.float32))
    p5 = fu._Plan(fu.BinaryOpNode("add_op", big, big2, (1 << 16, 1 << 16), np.float32), (1 << 16, 1 << 16), 4)
    assert p5.idx64


def test_cache_key_ignores_data_identity():
    def plan(ptr):
        x = fu.InputNode(FakeArray((1000,), np.float32, ptr=ptr))
        return fu._Plan(fu.UnaryOpNode("exp_op", x, (1000,), np.float32), (1000,), 4)
    assert plan(1 << 20).key() == plan(1 << 21).key()
    assert plan(1 << 20).key() != plan((1 << 20) + 4).key()  # alignment changes the code


def test_depth_tracking():
    x = fu.InputNode(FakeArray((10,), np.float32))
    n = x
    for _ in range(5):
        n = fu.UnaryOpNode("exp_op", n, (10,), np.float32)
    assert n._depth == 5
    assert fu._MAX_DEPTH == 16


def test_shard_threshold_config():
    """set_config(shard_threshold=...) (0 turns it off, negatives refused);
    without a multi-rank job nothing is sharded, whatever the threshold."""
    import numpy as np
    import pytest

    from macmetalpy_b200 import _config, distributed

    cfg = _config.get_config()
    try:
        _config.set_config(shard_threshold=100)
        assert cfg.shard_threshold == 100
        assert distributed._shard_host(np.ones(1000, np.float32), None, 100) is None  # not initialised
        _config.set_config(shard_threshold=0)
        assert cfg.shard_threshold is None
        with pytest.raises(ValueError):
            _config.set_config(shard_threshold=-1)
    finally:
        cfg.shard_threshold = None


def test_dist_operand_rules():
    """How a row-block DistArray lines its operands up with its block (host
    logic, numpy blocks standing in for device arrays): a DistArray of the
    same partition gives its block, an array spanning the global rows gives
    this rank's rows, a row-broadcast operand or a scalar passes unchanged,
    and a different partition is refused."""
    import numpy as np
    import pytest

    from macmetalpy_b200.distributed import DistArray

    g = np.arange(40.0).reshape(10, 4)
    a = DistArray(g[3:7], (10, 4), 3, 7)  # rows 3..6 of a 10-row array
    b = DistArray(g[3:7] * 2, (10, 4), 3, 7)
    np.testing.assert_array_equal(a._operand(b), g[3:7] * 2)
    np.testing.assert_array_equal(a._operand(g), g[3:7])
    row = np.ones((1, 4))
    assert a._operand(row) is row and a._operand(2.5) == 2.5
    with pytest.raises(ValueError):
        a._operand(DistArray(g[0:4], (10, 4), 0, 4))
    c = (a + g) * 2 - b
    assert isinstance(c, DistArray) and (c.start, c.stop, c.global_shape) == (3, 7, (10, 4))
    np.testing.assert_array_equal(c.local, 2 * g[3:7])  # (g + g) * 2 - 2g on the block
    s1 = a.map(lambda x: x.sum(axis=1))  # a per-row result keeps the row partition
    assert s1.global_shape == (10,) and s1.local.shape == (4,)
    assert a.ndim == 2 and a.size == 40
