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
