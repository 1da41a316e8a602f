"""Overlap of independent reductions on one stream (qsml_set_overlap).

A reduction that shares no buffer with the library kernels still running on
the stream starts reading at once and waits for them only at its end.  These
tests check that:
* a burst of independent reductions (every reduction kernel: segment, rows,
  columns, wide columns, split columns, strided lanes and column blocks)
  gives the same bits with overlap as without, eagerly and from a CUDA graph,
  and that the launches after the first did overlap;
* reductions that depend on one another (one reads what the previous wrote,
  or writes what the previous reads) wait, and give the right results;
* any other library kernel on the stream (an elementwise op) closes the
  window, so a reduction of its output waits for it.
"""
import numpy as np
import pytest

from helpers import d, dev, empty, host
from quasarml_b200 import abi, datagen

pytestmark = pytest.mark.gpu

# (shape, axis, dtype, kernel)
CASES = [((64, 512, 1024), None, np.float16, "k_reduce_seg"),
         ((64, 512, 1024), 2, np.float32, "k_reduce_rows"),
         ((64, 512, 1024), 1, np.float16, "k_reduce_cols"),
         ((64, 512, 1024), 0, np.float32, "k_reduce_cols_wide"),
         ((4096, 2048), 0, np.float32, "k_reduce_cols_split"),
         ((64, 512, 1024), 0, np.float16, "k_reduce_cols")]


def _inputs():
    import torch
    xs = []
    for i, (shape, axis, dt, _) in enumerate(CASES):
        x = dev(datagen.normal(70 + i, shape, 0.5, 1.0).astype(dt))
        tdt = torch.float32 if dt == np.float32 else torch.float16
        out = torch.empty(abi.reduced_shape(shape, axis, False), dtype=tdt, device="cuda")
        xs.append((x, out))
    # two strided views of one X[2048, 4096] fp32: rows along k, column blocks
    base = dev(datagen.normal(79, (2048, 4096), 0.5, 1.0))
    v = abi.make_desc(base.data_ptr() + (5 * 4096 + 1) * 4, abi.F32, (681, 2048), (3 * 4096, 2))
    o_rows = torch.empty((681,), device="cuda")
    o_cols = torch.empty((2048,), device="cuda")
    return xs, base, v, o_rows, o_cols


def _burst(ctx, xs, v, o_rows, o_cols, op):
    kernels = []
    for (x, out), (_, axis, _, _) in zip(xs, CASES):
        ctx.reduce(op, d(x), abi.AXIS_ALL if axis is None else axis, False, d(out))
        kernels.append(ctx.last_kernel())
    ctx.reduce(op, v, 1, False, d(o_rows))
    kernels.append(ctx.last_kernel())
    ctx.reduce(op, v, 0, False, d(o_cols))
    kernels.append(ctx.last_kernel())
    return kernels


def _results(xs, o_rows, o_cols):
    return [host(o).copy() for _, o in xs] + [host(o_rows).copy(), host(o_cols).copy()]


@pytest.mark.parametrize("op", [abi.RED_SUM, abi.RED_MEAN, abi.RED_MAX])
def test_independent_burst_same_bits(op):
    import torch
    xs, base, v, o_rows, o_cols = _inputs()
    ref_ctx = abi.Context(0)
    _burst(ref_ctx, xs, v, o_rows, o_cols, op)
    torch.cuda.synchronize()
    want = _results(xs, o_rows, o_cols)
    for _, o in xs:
        o.fill_(-7.0)
    o_rows.fill_(-7.0)
    o_cols.fill_(-7.0)

    ctx = abi.Context(0)
    ctx.set_overlap(True)
    p0, d0 = ctx.overlap_stats()
    kernels = _burst(ctx, xs, v, o_rows, o_cols, op)
    torch.cuda.synchronize()
    p1, d1 = ctx.overlap_stats()
    assert [c[3] for c in CASES] == kernels[:len(CASES)]
    assert kernels[-2:] == ["k_reduce_strided_lanes", "k_reduce_strided_cols"]
    assert p1 - p0 == len(kernels)
    assert d1 - d0 == len(kernels) - 1, "every launch after the first shares no buffer with those before it"
    got = _results(xs, o_rows, o_cols)
    for g, w, k in zip(got, want, kernels):
        assert np.array_equal(g.view(np.uint8), w.view(np.uint8)), k

    # the same burst captured in a CUDA graph and replayed
    for _, o in xs:
        o.fill_(-7.0)
    s = torch.cuda.Stream()
    ctx.set_stream(s.cuda_stream)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        _burst(ctx, xs, v, o_rows, o_cols, op)  # warm-up outside the graph
        s.synchronize()
        with torch.cuda.graph(g, stream=s):
            _burst(ctx, xs, v, o_rows, o_cols, op)
    for _ in range(3):
        for _, o in xs:
            o.fill_(-7.0)
        g.replay()
        torch.cuda.synchronize()
        got = _results(xs, o_rows, o_cols)
        for gg, w, k in zip(got, want, kernels):
            assert np.array_equal(gg.view(np.uint8), w.view(np.uint8)), k


def test_dependent_reductions_wait():
    """Read-after-write (a reduction of the previous one's output) and
    write-after-read (a reduction whose output lies in the bytes the previous
    one reads): each waits, over many rounds with no host sync in between."""
    import torch
    ctx = abi.Context(0)
    ctx.set_overlap(True)
    x = datagen.normal(81, (512, 8192), 0.5, 1.0)
    tx = dev(x)
    rows = empty((512,), np.float32)
    total = empty((1,), np.float32)
    y = datagen.normal(82, (1024, 4), 0.5, 1.0)
    ty = dev(y)
    want_rows = x.astype(np.float64).sum(axis=1)
    outs = []
    _, d0 = ctx.overlap_stats()
    for i in range(20):
        ctx.reduce(abi.RED_SUM, d(tx), 1, False, d(rows))          # reads X, writes rows
        ctx.reduce(abi.RED_SUM, d(rows), abi.AXIS_ALL, False, d(total))  # reads rows: waits
        t = empty((1,), np.float32)
        ctx.reduce(abi.RED_MAX, d(total), abi.AXIS_ALL, False, d(t))   # reads total: waits
        outs.append(t)
    torch.cuda.synchronize()
    _, d1 = ctx.overlap_stats()
    # the second and third reduction of a round read their predecessor's
    # output and wait; the first of the next round shares no buffer with the
    # third (the one kernel that may still run: it waited for the second) and
    # overlaps it
    assert d1 - d0 == 19
    for t in outs:
        assert abs(float(host(t)[0]) - want_rows.sum()) <= 1e-5 * np.abs(x).sum()

    # write-after-read: the second reduction's output is the first 4 KiB of X
    # while the first reduction reads all of X
    for _ in range(10):
        tx.copy_(torch.from_numpy(x).cuda())
        ctx.reduce(abi.RED_SUM, d(tx), 1, False, d(rows))
        over = abi.make_desc(tx.data_ptr(), abi.F32, (1024,), (1,))
        ctx.reduce(abi.RED_SUM, d(ty), 1, False, over)
        torch.cuda.synchronize()
        assert np.all(np.abs(host(rows).astype(np.float64) - want_rows) <= 1e-5 * np.abs(x).sum(axis=1))
        np.testing.assert_allclose(host(tx).reshape(-1)[:1024], y.sum(axis=1), rtol=1e-5)


def test_other_kernels_close_the_window():
    """A kernel that does not plan its launch (here qsml_fill) between two
    reductions closes the window: the reduction after it waits, and reads
    what it wrote.  An elementwise op plans its own launch: it overlaps an
    independent reduction before it, and a reduction of its output waits."""
    import torch
    ctx = abi.Context(0)
    ctx.set_overlap(True)
    a = dev(datagen.normal(83, (2048, 4096), 0.0, 1.0))
    b = dev(datagen.normal(84, (2048, 4096), 0.0, 1.0))
    s = empty((2048,), np.float32)
    first = empty((2048,), np.float32)
    for i in range(5):
        ctx.reduce(abi.RED_SUM, d(b), 1, False, d(first))
        ctx.fill(a.data_ptr(), np.float32(i + 1).tobytes(), a.numel())
        _, d0 = ctx.overlap_stats()
        ctx.reduce(abi.RED_SUM, d(a), 1, False, d(s))
        _, d1 = ctx.overlap_stats()
        assert d1 == d0
    torch.cuda.synchronize()
    assert np.all(host(s) == 5.0 * 4096)
    es = [torch.zeros((2048, 4096), device="cuda") for _ in range(5)]
    for e in es:
        ctx.reduce(abi.RED_SUM, d(b), 1, False, d(first))
        _, d0 = ctx.overlap_stats()
        ctx.binary_scalar(abi.OP_ADD, d(e), 1.0, d(e))  # e += 1: nothing in flight touches e
        _, d1 = ctx.overlap_stats()
        ctx.reduce(abi.RED_SUM, d(e), 1, False, d(s))  # reads e: waits
        _, d2 = ctx.overlap_stats()
        assert (d1 - d0, d2 - d1) == (1, 0)
    torch.cuda.synchronize()
    assert np.all(host(s) == 4096.0)


def test_long_burst_is_capped():
    """More independent reductions than the window holds: still right."""
    import torch
    ctx = abi.Context(0)
    ctx.set_overlap(True)
    xs = [dev(datagen.normal(90 + i, (256, 4096), 0.5, 1.0)) for i in range(40)]
    outs = [empty((256,), np.float32) for _ in xs]
    for x, o in zip(xs, outs):
        ctx.reduce(abi.RED_SUM, d(x), 1, False, d(o))
    torch.cuda.synchronize()
    p, dd = ctx.overlap_stats()
    assert 0 < dd < p
    for i, o in enumerate(outs):
        x = datagen.normal(90 + i, (256, 4096), 0.5, 1.0).astype(np.float64)
        assert np.all(np.abs(host(o) - x.sum(axis=1)) <= 1e-5 * np.abs(x).sum(axis=1))


def test_arg_reductions_overlap_same_indices():
    """argmax/argmin bursts (segment, rows and column kernels) give the same
    indices with overlap, and the launches after the first overlap."""
    import torch
    shapes = [((64, 512, 1024), None, np.float16), ((64, 512, 1024), 2, np.float32),
              ((64, 512, 1024), 1, np.float16), ((64, 512, 1024), 0, np.float32)]
    xs = [dev(datagen.normal(100 + i, s, 0.0, 1.0).astype(dt)) for i, (s, _, dt) in enumerate(shapes)]
    outs = [empty((1,) if ax is None else abi.reduced_shape(s, ax, False), np.int32) for s, ax, _ in shapes]

    def burst(ctx):
        names = []
        for op in (abi.ARG_MAX, abi.ARG_MIN):
            for x, o, (_, ax, _) in zip(xs, outs, shapes):
                ctx.arg_reduce(op, d(x), abi.AXIS_ALL if ax is None else ax, False, d(o))
                names.append(ctx.last_kernel())
        return names

    ref = abi.Context(0)
    burst(ref)
    torch.cuda.synchronize()
    want = [host(o).copy() for o in outs]
    for o in outs:
        o.fill_(-1)
    ctx = abi.Context(0)
    ctx.set_overlap(True)
    names = burst(ctx)
    torch.cuda.synchronize()
    p, dd = ctx.overlap_stats()
    assert names[:4] == ["k_arg_seg", "k_arg_rows", "k_arg_cols", "k_arg_cols"]
    # the second op's first launch writes what the first op's first launch
    # wrote (still in the window) and waits; the other six overlap
    assert (p, dd) == (8, 6)
    for g, w in zip([host(o) for o in outs], want):
        assert np.array_equal(g, w)


def test_row_ops_and_gathers_overlap_same_bits():
    """Layer norm, softmax and gathers of distinct tensors overlap like the
    reductions, with the same bits as without overlap."""
    import torch
    X32 = dev(datagen.normal(110, (16384, 4096), 0.5, 2.0))
    X16 = dev(datagen.normal(111, (16384, 4096), 0.5, 2.0).astype(np.float16))
    g = dev(datagen.normal(112, (4096,), 1.0, 0.1))
    b = dev(datagen.normal(113, (4096,), 0.0, 0.1))
    G = dev(datagen.uniform(114, (8192, 8192), -1, 1))
    v1 = abi.make_desc(G.data_ptr() + (5 * 8192 + 1) * 4, abi.F32, (2729, 4096), (3 * 8192, 2))
    v2 = abi.make_desc(G.data_ptr(), abi.F32, (2048, 8192), (4, 8192))
    outs = [torch.empty_like(X32), torch.empty_like(X16), torch.empty_like(X32), torch.empty_like(X16),
            torch.empty((2729, 4096), device="cuda"), torch.empty((2048, 8192), device="cuda")]

    def burst(ctx):
        names = []
        ctx.layer_norm(d(X32), d(g), d(b), 1e-5, d(outs[0]))
        names.append(ctx.last_kernel())
        ctx.layer_norm(d(X16), d(g), d(b), 1e-5, d(outs[1]))
        names.append(ctx.last_kernel())
        ctx.softmax(d(X32), -1, d(outs[2]))
        names.append(ctx.last_kernel())
        ctx.softmax(d(X16), -1, d(outs[3]))
        names.append(ctx.last_kernel())
        ctx.gather(v1, d(outs[4]))
        names.append(ctx.last_kernel())
        ctx.gather(v2, d(outs[5]))
        names.append(ctx.last_kernel())
        return names

    ref = abi.Context(0)
    burst(ref)
    torch.cuda.synchronize()
    want = [host(o).copy() for o in outs]
    for o in outs:
        o.zero_()
    ctx = abi.Context(0)
    ctx.set_overlap(True)
    names = burst(ctx)
    torch.cuda.synchronize()
    p, dd = ctx.overlap_stats()
    assert (p, dd) == (6, 5), names
    for gg, w, k in zip([host(o) for o in outs], want, names):
        assert np.array_equal(gg.view(np.uint8), w.view(np.uint8)), k


def test_fused_kernels_overlap_and_readers_wait():
    """Runtime-compiled fused kernels of distinct batch entries overlap; a
    reduction of a fused kernel's output waits for it (read-after-write)."""
    import torch
    A = [dev(datagen.uniform(120 + i, (4096, 4096), -1.0, 1.0)) for i in range(4)]
    B = dev(datagen.uniform(125, (1, 4096), -1.0, 1.0))
    D = dev(datagen.uniform(126, (4096, 1), 0.5, 2.0))
    outs = [empty((4096, 4096), np.float32) for _ in A]
    sums = [empty((4096,), np.float32) for _ in A]
    e = abi.Expr()
    a, b, dd = e.input(0), e.input(1), e.input(2)
    t = e.binary(abi.OP_SUB, e.binary(abi.OP_MUL, e.binary(abi.OP_ADD, a, b), b), a)
    e.unary(abi.UN_RELU, e.binary(abi.OP_DIV, e.binary(abi.OP_POW, t, e.const(2.0)), dd))

    def run(ctx, with_sums):
        for i in range(4):
            ctx.elementwise_fused(e.nodes, [d(A[i]), d(B), d(D)], d(outs[i]))
            if with_sums:
                ctx.reduce(abi.RED_SUM, d(outs[i]), 1, False, d(sums[i]))

    ref = abi.Context(0)
    ref.set_fuse_mode(abi.FUSE_MODE_JIT)
    run(ref, True)
    torch.cuda.synchronize()
    want = [host(o).copy() for o in outs]
    want_s = [host(s).copy() for s in sums]
    for o in outs + sums:
        o.zero_()
    ctx = abi.Context(0)
    ctx.set_fuse_mode(abi.FUSE_MODE_JIT)
    ctx.set_overlap(True)
    run(ctx, False)  # four independent fused kernels
    torch.cuda.synchronize()
    p, dd0 = ctx.overlap_stats()
    assert (p, dd0) == (4, 3)
    for o in outs:
        o.zero_()
    run(ctx, True)  # each reduction reads the fused kernel just before it
    torch.cuda.synchronize()
    for g, w in zip([host(o) for o in outs], want):
        assert np.array_equal(g.view(np.uint32), w.view(np.uint32))
    for g, w in zip([host(s) for s in sums], want_s):
        assert np.array_equal(g.view(np.uint32), w.view(np.uint32))


def _random_program(seed, nops):
    """A seeded sequence of ops over a pool of 6 buffers of [1024, 1024]
    binary32, each op reading and writing 256-row blocks (or whole buffers)
    chosen at random, so that reads-after-writes, writes-after-reads and
    writes-after-writes between consecutive and nearby ops are frequent."""
    rng = np.random.default_rng(seed)
    prog = []
    for _ in range(nops):
        kind = rng.choice(["red_rows", "red_cols", "red_all", "arg_rows", "gather_t", "layer_norm", "softmax",
                           "add", "fused"])
        src, dst = int(rng.integers(6)), int(rng.integers(6))
        qs, qd = int(rng.integers(4)), int(rng.integers(4))
        if kind in ("gather_t", "red_rows", "red_cols", "red_all", "arg_rows") and src == dst:
            dst = (dst + 1) % 6  # no kernel writes into what it reads
        if kind in ("layer_norm", "softmax", "fused", "add") and src == dst and qs == qd:
            qd = (qd + 1) % 4
        prog.append((str(kind), src, dst, qs, qd, int(rng.integers(6)), int(rng.integers(2))))
    return prog


def _run_program(ctx, pool, g, b, prog):
    import torch
    R, C = 256, 1024
    blk = R * C

    def view(i, q, rows=R):
        return abi.make_desc(pool[i].data_ptr() + q * blk * 4, abi.F32, (rows, C), (C, 1))

    e = abi.Expr()
    x0, x1 = e.input(0), e.input(1)
    e.binary(abi.OP_ADD, e.binary(abi.OP_MUL, x0, e.const(0.5)), e.unary(abi.UN_RELU, x1))
    for kind, src, dst, qs, qd, other, opbit in prog:
        op = abi.RED_MAX if opbit else abi.RED_MEAN
        if kind == "red_rows":
            out = abi.make_desc(pool[dst].data_ptr() + qd * blk * 4, abi.F32, (R,), (1,))
            ctx.reduce(op, view(src, qs), 1, False, out)
        elif kind == "red_cols":
            out = abi.make_desc(pool[dst].data_ptr() + qd * blk * 4, abi.F32, (C,), (1,))
            ctx.reduce(op, view(src, qs), 0, False, out)
        elif kind == "red_all":
            out = abi.make_desc(pool[dst].data_ptr() + (qd * blk + 7) * 4, abi.F32, (1,), (1,))
            ctx.reduce(op, abi.make_desc(pool[src].data_ptr(), abi.F32, (1024, C), (C, 1)), abi.AXIS_ALL, False, out)
        elif kind == "arg_rows":
            out = abi.make_desc(pool[dst].data_ptr() + qd * blk * 4, abi.I32, (R,), (1,))
            ctx.arg_reduce(abi.ARG_MAX if opbit else abi.ARG_MIN, view(src, qs), 1, False, out)
            # the indices land as floats' bits: small integers, harmless inputs
        elif kind == "gather_t":
            t = abi.make_desc(pool[src].data_ptr(), abi.F32, (1024, C), (1, C))
            ctx.gather(t, abi.make_desc(pool[dst].data_ptr(), abi.F32, (1024, C), (C, 1)))
        elif kind == "layer_norm":
            ctx.layer_norm(view(src, qs), d(g), d(b), 1e-5, view(dst, qd))
        elif kind == "softmax":
            ctx.softmax(view(src, qs), -1, view(dst, qd))
        elif kind == "add":
            ctx.binary(abi.OP_ADD, view(src, qs), view(other, (qs + 1) % 4), view(dst, qd))
        else:
            ctx.elementwise_fused(e.nodes, [view(src, qs), view(other, qd)], view(dst, (qd + 2) % 4))
    torch.cuda.synchronize()


@pytest.mark.parametrize("seed", [1, 2, 3])
def test_random_programs_same_bits_with_overlap(seed):
    """Seeded random programs of reductions, arg-reductions, gathers, layer
    norms, softmaxes, adds and fused expressions over a small pool of
    buffers, so that dependent and independent neighbours mix: with overlap
    on, every buffer ends bit-identical to the run without it."""
    import torch
    init = [datagen.uniform(200 + i, (1024, 1024), -1.0, 1.0) for i in range(6)]
    g = dev(datagen.normal(210, (1024,), 1.0, 0.1))
    b = dev(datagen.normal(211, (1024,), 0.0, 0.1))
    prog = _random_program(seed, 300)
    results = []
    for overlap in (False, True):
        pool = [dev(x) for x in init]
        ctx = abi.Context(0)
        ctx.set_overlap(overlap)
        _run_program(ctx, pool, g, b, prog)
        results.append([host(p).copy() for p in pool])
        if overlap:
            planned, deferred = ctx.overlap_stats()
            assert deferred > 0, (planned, deferred)
    for i, (r0, r1) in enumerate(zip(*results)):
        assert np.array_equal(r0.view(np.uint32), r1.view(np.uint32)), f"buffer {i}"
