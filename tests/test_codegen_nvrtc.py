"""The fusion emitter produces CUDA C that NVRTC compiles for sm_100a.

Runs on CPU: graphs are built over stand-in arrays (pointer, shape, strides,
dtype only) and the generated elementwise and reduction kernels are compiled
with NVRTC through cuda-python, with the options the library uses.
"""

import numpy as np
import pytest

from macmetalpy_b200 import _fusion as fu

nvrtc = pytest.importorskip("cuda.bindings.nvrtc")


class FakeArray:
    def __init__(self, shape, dtype, strides=None, ptr=1 << 20, offset=0):
        self._shape = tuple(shape)
        self._dtype = np.dtype(dtype)
        self._strides = tuple(strides) if strides is not None else fu._c_strides(self._shape)
        self._ptr = ptr + offset * self._dtype.itemsize
        self._offset = 0
        self._fusion_node = None


def _compile(src: str, name: str):
    opts = [o for o in fu._options().decode().split("\n") if o]
    rc, prog = nvrtc.nvrtcCreateProgram(src.encode(), b"t.cu", 0, [], [])
    assert rc == nvrtc.nvrtcResult.NVRTC_SUCCESS
    rc2, = nvrtc.nvrtcCompileProgram(prog, len(opts), [o.encode() for o in opts])
    if rc2 != nvrtc.nvrtcResult.NVRTC_SUCCESS:
        _, n = nvrtc.nvrtcGetProgramLogSize(prog)
        log = b" " * n
        nvrtc.nvrtcGetProgramLog(prog, log)
        pytest.fail(f"NVRTC failed for {name}:\n{log.decode(errors='replace')}\n{src}")


def _inp(shape, dtype, **kw):
    return fu.InputNode(FakeArray(shape, dtype, **kw))


def _c1_expr(n=1 << 20):
    x = _inp((n,), np.float32)
    ab = fu.UnaryOpNode("abs_op", x, (n,), np.float32)
    sq = fu.UnaryOpNode("sqrt_op", ab, (n,), np.float32)
    x2 = fu.UnaryOpNode("square_op", x, (n,), np.float32)
    ng = fu.UnaryOpNode("neg_op", x2, (n,), np.float32)
    ex = fu.UnaryOpNode("exp_op", ng, (n,), np.float32)
    return fu.BinaryOpNode("add_op", sq, ex, (n,), np.float32)


CASES = {
    "c1_expression": lambda: (_c1_expr(), (1 << 20,)),
    "binary_f32": lambda: (fu.BinaryOpNode("floor_divide_op", _inp((1000,), np.float32), _inp((1000,), np.float32),
                                           (1000,), np.float32), (1000,)),
    "binary_i32_mod": lambda: (fu.BinaryOpNode("mod_op", _inp((1000,), np.int32), _inp((1000,), np.int32),
                                               (1000,), np.int32), (1000,)),
    "logaddexp": lambda: (fu.BinaryOpNode("logaddexp_op", _inp((1000,), np.float32), _inp((1000,), np.float32),
                                          (1000,), np.float32), (1000,)),
    "broadcast_rows_cols": lambda: (fu.BinaryOpNode("add_op", _inp((8192, 1), np.float32),
                                                    _inp((1, 32768), np.float32), (8192, 32768), np.float32),
                                    (8192, 32768)),
    "strided_transpose": lambda: (fu.UnaryOpNode("exp_op", _inp((64, 32), np.float32, strides=(1, 64)),
                                                 (64, 32), np.float32), (64, 32)),
    "scalar_f16": lambda: (fu.BinaryOpNode("mul_op", _inp((100,), np.float16), fu.ScalarNode(3.0, np.float16),
                                           (100,), np.float16), (100,)),
    "cast_chain": lambda: (fu.CastNode(fu.BinaryOpNode("add_op", _inp((77,), np.int16), _inp((77,), np.int16),
                                                       (77,), np.int16), np.float64), (77,)),
    "compare_select": lambda: (fu.SelectNode(fu.BinaryOpNode("gt_op", _inp((50,), np.float32),
                                                             fu.ScalarNode(0, np.float32), (50,), np.bool_,
                                                             in_dtype=np.float32),
                                             _inp((50,), np.float32), fu.ScalarNode(0, np.float32), (50,),
                                             np.float32), (50,)),
    "huge_idx64": lambda: (fu.BinaryOpNode("add_op", _inp((1 << 16, 1), np.float32),
                                           _inp((1, 1 << 16), np.float32), (1 << 16, 1 << 16), np.float32),
                           (1 << 16, 1 << 16)),
    "all_unary": lambda: (_unary_chain(), (256,)),
    "all_binary": lambda: (_binary_chain(), (256,)),
    "int_bits_i32": lambda: (_int_bits_chain(np.int32), (256,)),
    "int_bits_u8": lambda: (_int_bits_chain(np.uint8), (256,)),
    "int_bits_i64": lambda: (_int_bits_chain(np.int64), (256,)),
    "predicates_logic": lambda: (_predicates(), (256,)),
}


_INT_ONLY = {"invert_op", "bitwise_and_op", "bitwise_or_op", "bitwise_xor_op", "left_shift_op", "right_shift_op"}


def _unary_chain():
    node = _inp((256,), np.float32)
    for op in sorted(fu._FUSEABLE_UNARY_OPS - _INT_ONLY):
        node = fu.UnaryOpNode(op, node, (256,), np.float32)
    return node


def _binary_chain():
    a = _inp((256,), np.float64)
    node = a
    for op in sorted(fu._FUSEABLE_BINARY_OPS - _INT_ONLY):
        if op in fu._CMP:
            continue
        node = fu.BinaryOpNode(op, node, a, (256,), np.float64)
    return node


def _int_bits_chain(dt=np.int32):
    a = _inp((256,), dt)
    b = _inp((256,), dt)
    node = a
    for op in sorted(_INT_ONLY - {"invert_op"}):
        node = fu.BinaryOpNode(op, node, b, (256,), dt)
    return fu.UnaryOpNode("invert_op", node, (256,), dt)


def _predicates():
    x = _inp((256,), np.float32)
    n = (256,)
    p = [fu.UnaryOpNode(op, x, n, np.bool_, in_dtype=np.float32)
         for op in ("isnan_op", "isinf_op", "isfinite_op", "signbit_op", "logical_not_op")]
    node = p[0]
    for q, op in zip(p[1:], ("logical_and_op", "logical_or_op", "logical_xor_op", "logical_and_op")):
        node = fu.BinaryOpNode(op, node, q, n, np.bool_, in_dtype=np.bool_)
    return fu.BinaryOpNode("logical_or_op", node, x, n, np.bool_, in_dtype=np.float32)


@pytest.mark.parametrize("case", sorted(CASES))
def test_elementwise_source_compiles(case):
    node, shape = CASES[case]()
    plan = fu._Plan(node, shape, 4)
    _compile(fu._ew_source(plan, False), case)


@pytest.mark.parametrize("opc", [0, 4, 5, 7, 9, 10])
def test_fused_reduce_source_compiles(opc):
    node, shape = _c1_expr(), (1 << 20,)
    plan = fu._Plan(node, shape, 4)
    _compile(fu._red_source(plan, opc, "full", 1), f"reduce{opc}")


@pytest.mark.parametrize("kind", ["rows_block", "rows_warp", "cols"])
def test_fused_axis_reduce_source_compiles(kind):
    x = _inp((128, 256), np.float32)
    node = fu.UnaryOpNode("exp_op", x, (128, 256), np.float32)
    plan = fu._Plan(node, (128, 256), 4)
    _compile(fu._red_source(plan, 5, kind, 4 if kind == "cols" else 1), kind)


def test_strided_output_source_compiles():
    node, shape = _c1_expr(1000), (1000,)
    plan = fu._Plan(node, shape, 4)
    plan.strided = True
    plan.nd = 1
    plan.cshape = [1000]
    plan.cstrides = [[1]]
    plan.kinds = ["sg"]
    plan.vec_ok = False
    plan.idx64 = True
    _compile(fu._ew_source(plan, True), "strided_out")


def test_fastdiv_matches_integer_division():
    rng = np.random.default_rng(0)
    for d in list(range(1, 70)) + [int(v) for v in rng.integers(1, 1 << 31, 200)]:
        m, s = fu._fastdiv(d)
        for n in [0, 1, d - 1, d, d + 1, (1 << 32) - 1, (1 << 31)] + [int(v) for v in rng.integers(0, 1 << 32, 50)]:
            q = (((n * m) >> 32) + n) >> s
            assert q == n // d, (n, d)
