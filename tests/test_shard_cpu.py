"""CPU tests of the row-sharded classifier's host logic: partitioning, and a
world-size-2 gloo all-gather whose gathered logits (computed per shard by the
oracle) are bit-identical to the single-process result, argmax included."""
import os
import socket

import numpy as np
import pytest

from minillama_infra_b200.shard import row_shard


@pytest.mark.parametrize("d,world", [(128256, 1), (128256, 2), (128256, 8), (10, 3), (7, 8), (1, 4)])
def test_row_shards_cover_rows_once(d, world):
    seen = []
    for r in range(world):
        s = row_shard(d, world, r)
        assert s.rows >= 0 and s.rows <= s.chunk
        seen.extend(range(s.r0, s.r1))
    assert seen == list(range(d))


def test_row_shard_rejects_bad_requests():
    for args in [(0, 2, 0), (10, 0, 0), (10, 2, 2), (10, 2, -1)]:
        with pytest.raises(ValueError):
            row_shard(*args)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, d, n, form, q):
    import torch
    import torch.distributed as dist

    from minillama_infra_b200.shard import ShardedLinear
    from minillama_infra_b200 import synth
    from oracle import oracle as orc

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w_q, w_s = orc.quantize_weights(synth.weights_np(d, n, 11))
        x = synth.activation_np(n, 12, outliers=(form == "w8a8"))
        s = row_shard(d, world, rank)

        def compute(y, xt):
            xs = xt.numpy()
            if form == "w8a32":
                out = orc.gemv_w8a32(xs, w_q[s.r0:s.r1], w_s[s.r0:s.r1])
            else:
                xq, xsc = orc.quantize_activation(xs)
                out = orc.gemv_w8a8(xq, xsc, w_q[s.r0:s.r1], w_s[s.r0:s.r1])
            y.copy_(torch.from_numpy(out))

        lin = ShardedLinear(torch.from_numpy(w_q[s.r0:s.r1]), torch.from_numpy(w_s[s.r0:s.r1]),
                            d, n, rank, world, form=form, compute=compute)
        logits = lin.forward(torch.from_numpy(x)).numpy().copy()
        if rank == 0:
            q.put(logits)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("form", ["w8a32", "w8a8"])
@pytest.mark.parametrize("d", [1000, 1001])
def test_gloo_allgather_matches_single_process(form, d):
    import torch.multiprocessing as mp

    from minillama_infra_b200 import synth
    from oracle import oracle as orc

    n, world = 512, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, d, n, form, q)) for r in range(world)]
    for p in procs:
        p.start()
    gathered = q.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    w_q, w_s = orc.quantize_weights(synth.weights_np(d, n, 11))
    x = synth.activation_np(n, 12, outliers=(form == "w8a8"))
    if form == "w8a32":
        ref = orc.gemv_w8a32(x, w_q, w_s)
    else:
        xq, xs = orc.quantize_activation(x)
        ref = orc.gemv_w8a8(xq, xs, w_q, w_s)
    assert np.array_equal(gathered.view(np.uint32), ref.view(np.uint32))
    assert int(np.argmax(gathered)) == int(np.argmax(ref))


def _silu_mul(g, u):
    g = g.astype(np.float32)
    return ((g * (np.float32(1.0) / (np.float32(1.0) + np.exp(-g)))) * u).astype(np.float32)


def _ffn_ref(x, gate, up, down, form, rows=None, drows=None):
    """The FFN block on the CPU (oracle GEMVs) over gate/up rows `rows` and down rows `drows`."""
    from oracle import oracle as orc

    def gemv(xv, q, s):
        if form == "w8a32":
            return orc.gemv_w8a32(xv, q, s)
        xq, xs = orc.quantize_activation(xv)
        return orc.gemv_w8a8(xq, xs, q, s)

    rows = slice(None) if rows is None else rows
    drows = slice(None) if drows is None else drows
    hb = _silu_mul(gemv(x, gate[0][rows], gate[1][rows]), gemv(x, up[0][rows], up[1][rows]))
    return hb, (lambda hb_full: gemv(hb_full, down[0][drows], down[1][drows]))


def _ffn_weights(dim, hidden):
    from minillama_infra_b200 import synth
    from oracle import oracle as orc

    gate = orc.quantize_weights(synth.weights_np(hidden, dim, 21))
    up = orc.quantize_weights(synth.weights_np(hidden, dim, 22))
    down = orc.quantize_weights(synth.weights_np(dim, hidden, 23))
    return gate, up, down


def _ffn_worker(rank, world, port, dim, hidden, form, q):
    import torch
    import torch.distributed as dist

    from minillama_infra_b200 import synth
    from minillama_infra_b200.shard import ShardedFFN

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        gate, up, down = _ffn_weights(dim, hidden)
        x = synth.activation_np(dim, 24, outliers=(form == "w8a8"))
        hs, ds = row_shard(hidden, world, rank), row_shard(dim, world, rank)
        hb_local, down_fn = _ffn_ref(x, gate, up, down, form, slice(hs.r0, hs.r1), slice(ds.r0, ds.r1))

        def gateup(y, xt):
            y.copy_(torch.from_numpy(hb_local))

        def down_c(y, hb):
            y.copy_(torch.from_numpy(down_fn(hb.numpy())))

        t = lambda a: torch.from_numpy(np.ascontiguousarray(a))  # noqa: E731
        ffn = ShardedFFN(t(gate[0][hs.r0:hs.r1]), t(gate[1][hs.r0:hs.r1]), t(up[0][hs.r0:hs.r1]),
                         t(up[1][hs.r0:hs.r1]), t(down[0][ds.r0:ds.r1]), t(down[1][ds.r0:ds.r1]),
                         dim, hidden, rank, world, form=form, compute_gateup=gateup, compute_down=down_c)
        xb = ffn.forward(torch.from_numpy(x)).numpy().copy()
        hb = ffn.hidden_vector().numpy().copy()
        if rank == 0:
            q.put((hb, xb))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("form", ["w8a32", "w8a8"])
@pytest.mark.parametrize("dim,hidden", [(256, 1024), (192, 640)])
def test_gloo_ffn_shard_matches_single_process(form, dim, hidden):
    """gate/up row shards -> all-gather hb -> down row shards -> all-gather xb,
    bit-identical to the whole block on one process."""
    import torch.multiprocessing as mp

    from minillama_infra_b200 import synth

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ffn_worker, args=(r, world, port, dim, hidden, form, q)) for r in range(world)]
    for p in procs:
        p.start()
    hb, xb = q.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    gate, up, down = _ffn_weights(dim, hidden)
    x = synth.activation_np(dim, 24, outliers=(form == "w8a8"))
    hb_ref, down_fn = _ffn_ref(x, gate, up, down, form)
    assert np.array_equal(hb.view(np.uint32), hb_ref.view(np.uint32))
    assert np.array_equal(xb.view(np.uint32), down_fn(hb_ref).view(np.uint32))


def test_ffn_shard_rejects_wrong_shapes():
    import torch

    from minillama_infra_b200.shard import ShardedFFN

    z8 = lambda r, c: torch.zeros((r, c), dtype=torch.int8)  # noqa: E731
    zs = lambda r, c: torch.zeros((r, c // 64), dtype=torch.float32)  # noqa: E731
    with pytest.raises(ValueError):  # gate shard of the wrong row count for rank 0 of 2
        ShardedFFN(z8(100, 256), zs(100, 256), z8(512, 256), zs(512, 256), z8(128, 1024), zs(128, 1024),
                   256, 1024, 0, 2)
    with pytest.raises(ValueError):
        ShardedFFN(z8(512, 256), zs(512, 256), z8(512, 256), zs(512, 256), z8(128, 1024), zs(128, 1024),
                   256, 1024, 0, 2, form="fp16")
