"""Transpose materialisation on the device, bit for bit.

4-byte element types with row lengths divisible by 4 take the vectorised
64 x 64 tile kernel; everything else the 32 x 32 scalar kernel.  Both must
return what the oracle returns (codegen.c:363-369: x.T; f16 graphs pass
through the emitter's own f16 <-> f32 conversions, which rescale f16
subnormals), on whole and ragged tile edges."""
import numpy as np
import pytest

import bafe_b200 as bafe
from bafe_b200.graph import GraphBuilder
from oracle import oracle

pytestmark = pytest.mark.gpu

DT = {np.float32: 0, np.float64: 1, np.int32: 2, np.float16: 4}


def _transpose(x):
    g = GraphBuilder()
    xi = g.add_input("X", x.shape, DT[x.dtype.type], 0)
    g.set_output(g.add("transpose", [xi], perm=[1, 0]))
    k = bafe.compile_graph(g)
    want = oracle.evaluate(g.to_list(), {xi: x}, g.output).reshape(x.shape[::-1])
    return k(x), k.describe(), want


@pytest.mark.parametrize("shape", [(4, 8), (64, 64), (68, 132), (196, 260), (1000, 4), (4100, 4096), (37, 53),
                                   (1, 1000), (130, 3)])
@pytest.mark.parametrize("dtype", [np.float32, np.int32, np.float64, np.float16])
def test_transpose_is_exact(cuda, shape, dtype):
    rng = np.random.default_rng(hash((shape, dtype.__name__)) % (1 << 32))
    if np.issubdtype(dtype, np.integer):
        x = rng.integers(-2**31, 2**31 - 1, size=shape, dtype=dtype)
    else:
        x = rng.standard_normal(shape).astype(dtype)
    out, plan, want = _transpose(x)
    assert "transpose2d" in plan
    assert out.shape == shape[::-1]
    assert out.tobytes() == want.tobytes()
    if dtype != np.float16:
        assert out.tobytes() == np.ascontiguousarray(x.T).tobytes()


def test_transpose_of_special_values_is_a_bit_copy(cuda):
    x = np.array([[np.nan, -0.0, np.inf, -np.inf], [1e-45, -1e-45, 3.0, -3.0],
                  [0.0, 1.0, 2.0, 3.0], [4.0, 5.0, 6.0, 7.0]], np.float32)
    x.view(np.uint32)[0, 0] = 0x7FC12345              # NaN payload survives
    out, _, _ = _transpose(x)
    assert out.view(np.uint32).tobytes() == np.ascontiguousarray(x.T).view(np.uint32).tobytes()


@pytest.mark.parametrize("shape,perm", [
    ((3, 68, 132), (0, 2, 1)),         # batch of 16-byte-kernel transposes
    ((5, 37, 53), (0, 2, 1)),          # scalar kernel, ragged tiles
    ((2, 3, 64, 40), (0, 1, 3, 2)),    # two leading axes
    ((4, 6, 8), (1, 0, 2)),            # other permutation: the strided gather
])
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_rank_n_transpose_is_exact(cuda, shape, perm, dtype):
    """Swapping the last two axes runs as a batch of tiled rank-2 transposes;
    other permutations take the strided gather.  Bit copies either way."""
    rng = np.random.default_rng(sum(shape) + len(perm))
    x = rng.standard_normal(shape).astype(dtype)
    g = GraphBuilder()
    xi = g.add_input("X", x.shape, DT[x.dtype.type], 0)
    g.set_output(g.add("transpose", [xi], perm=list(perm)))
    k = bafe.compile_graph(g)
    swap_last = tuple(perm[:-2]) == tuple(range(len(perm) - 2)) and tuple(perm[-2:]) == (len(perm) - 1, len(perm) - 2)
    assert ("transpose2d" in k.describe()) == swap_last, k.describe()
    out = k(x)
    assert out.tobytes() == np.ascontiguousarray(np.transpose(x, perm)).tobytes()


@pytest.mark.parametrize("shape,perm", [
    ((4, 6, 8), (1, 0, 2)),            # innermost axis kept, length % 4 == 0: vector gather
    ((16, 64, 128), (1, 0, 2)),
    ((2, 3, 4, 8), (2, 0, 1, 3)),
    ((3, 5, 7), (1, 0, 2)),            # length 7: element gather
])
@pytest.mark.parametrize("dtype", [np.float32, np.float64, np.float16])
def test_gather_transposes_keeping_the_last_axis(cuda, shape, perm, dtype):
    rng = np.random.default_rng(sum(shape))
    x = rng.standard_normal(shape).astype(dtype)
    g = GraphBuilder()
    xi = g.add_input("X", x.shape, DT[x.dtype.type], 0)
    g.set_output(g.add("transpose", [xi], perm=list(perm)))
    k = bafe.compile_graph(g)
    want = oracle.evaluate(g.to_list(), {xi: x}, g.output).reshape(np.transpose(x, perm).shape)
    out = k(x)
    assert out.tobytes() == want.tobytes()
    if dtype != np.float16:
        assert out.tobytes() == np.ascontiguousarray(np.transpose(x, perm)).tobytes()


@pytest.mark.parametrize("src,dst", [((8,), (3, 8)), ((1, 12), (5, 12)), ((5, 1), (5, 8)), ((2, 1, 16), (2, 3, 16))])
def test_broadcast_to(cuda, src, dst):
    rng = np.random.default_rng(len(dst))
    x = rng.standard_normal(src).astype(np.float32)
    g = GraphBuilder()
    xi = g.add_input("X", src, 0, 0)
    g.set_output(g.add("broadcast_to", [xi], shape=list(dst)))
    out = bafe.compile_graph(g)(x)
    assert out.tobytes() == np.ascontiguousarray(np.broadcast_to(x, dst)).tobytes()


@pytest.mark.parametrize("shape,perm", [
    ((70000, 3, 5), (0, 2, 1)),        # scalar kernel, 70000 items: two launches of <= 65535
    ((66000, 4, 8), (0, 2, 1)),        # 16-byte kernel, 66000 items
    ((3, 2100000), (1, 0)),            # scalar kernel, 65625 row tiles of 32
    ((4, 4200000), (1, 0)),            # 16-byte kernel, 65625 row tiles of 64
])
def test_transpose_beyond_one_grid(cuda, shape, perm):
    """A grid's y and z stop at 65535: more batch items or row tiles than
    that run as several launches, with the same bits as one would give.
    Device-resident call, so that no host row panel splits the problem."""
    torch = cuda
    g = GraphBuilder()
    xi = g.add_input("X", shape, 0, 0)
    g.set_output(g.add("transpose", [xi], perm=list(perm)))
    k = bafe.compile_graph(g)
    assert "transpose2d" in k.describe()
    gen = torch.Generator(device="cuda").manual_seed(7)
    x = torch.randn(shape, device="cuda", generator=gen)
    out = torch.empty(x.numel(), device="cuda")
    before = bafe.launch_count()
    k.run_torch([x], out)
    torch.cuda.synchronize()
    assert bafe.launch_count() - before == 2
    assert torch.equal(out, x.permute(*perm).contiguous().reshape(-1))
