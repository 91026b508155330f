"""Multi-GPU row-sharded classifier on real GPUs (NCCL), run when the box has
at least two: every rank's gathered logits are bit-identical to the
single-GPU GEMV of the whole matrix, and so is the argmax."""
import os
import socket

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, d, n, form, q, fused=False):
    from datetime import timedelta

    import torch.distributed as dist

    from minillama_infra_b200 import ops, synth
    from minillama_infra_b200.shard import ShardedLinear, row_shard

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    try:
        w_q, w_s = synth.weights_gpu(d, n, seed=99, device=dev)
        x = synth.activation_gpu(n, 7, dev, outliers=(form == "w8a8"))
        sh = row_shard(d, world, rank)
        full = torch.empty(d, dtype=torch.float32, device=dev)
        if form == "w8a32":
            ops.matmul_int8(full, x, w_q, w_s, n, d, 64)
        else:
            ops.matmul_dp4a_fused(full, x, w_q, w_s, n, d, 64)
        want = int(torch.argmax(full).item())
        if not fused:
            lin = ShardedLinear(w_q[sh.r0:sh.r1].clone(), w_s[sh.r0:sh.r1].clone(), d, n, rank, world, form=form)
            logits = lin.forward(x)
            torch.cuda.synchronize()
            same = bool(torch.equal(logits.view(torch.int32), full.view(torch.int32)))
            arg = int(torch.argmax(logits).item()) == want
        else:
            from minillama_infra_b200.shard import PeerShardedLinear

            lin = PeerShardedLinear(w_q[sh.r0:sh.r1].clone(), w_s[sh.r0:sh.r1].clone(), d, n, rank, world,
                                    form=form)
            same, arg = True, True
            full_bits = full.cpu().numpy().view("uint32")
            given = torch.full((), -1, dtype=torch.int64, device=dev)
            for step in range(5):  # both logits halves, several times
                # odd steps write the argmax into a tensor of the caller's
                out = lin.forward(x, out=given) if step % 2 else lin.forward(x)
                torch.cuda.synchronize()
                dist.barrier()  # every rank's words of this step have landed
                got = lin.read_logits(step)  # also checks every word's step tag
                same = same and bool((got.view("uint32") == full_bits).all())
                arg = arg and int(out.item()) == want and (out is given) == (step % 2 == 1)
                dist.barrier()
            lin.close()
        q.put((rank, same, arg, ops.device_error()))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("form", ["w8a32", "w8a8"])
def test_peer_sharded_classifier_one_gpu(form):
    """world == 1: the fused GEMV + argmax without a process group, the argmax
    written into the tensor given to forward() and the logits bit-exact."""
    from minillama_infra_b200 import ops, synth
    from minillama_infra_b200.shard import PeerShardedLinear

    dev = torch.device("cuda", 0)
    d, n = 128256 // 8 + 3, 2048
    w_q, w_s = synth.weights_gpu(d, n, seed=99, device=dev)
    x = synth.activation_gpu(n, 7, dev, outliers=(form == "w8a8"))
    full = torch.empty(d, dtype=torch.float32, device=dev)
    if form == "w8a32":
        ops.matmul_int8(full, x, w_q, w_s, n, d, 64)
    else:
        ops.matmul_dp4a_fused(full, x, w_q, w_s, n, d, 64)
    want = int(torch.argmax(full).item())
    lin = PeerShardedLinear(w_q, w_s, d, n, 0, 1, form=form)
    given = torch.full((), -1, dtype=torch.int64, device=dev)
    try:
        for step in range(3):
            out = lin.forward(x, out=given)
            torch.cuda.synchronize()
            assert out is given and int(given.item()) == want
            got = lin.read_logits(step)
            assert (got.view("uint32") == full.cpu().numpy().view("uint32")).all()
        with pytest.raises(ValueError):
            lin.forward(x, out=torch.zeros(2, dtype=torch.int64, device=dev))
        assert ops.device_error() == 0
    finally:
        lin.close()


@pytest.mark.parametrize("fused", [False, True], ids=["nccl", "p2p"])
@pytest.mark.parametrize("form", ["w8a32", "w8a8"])
def test_sharded_classifier_bit_exact_two_gpus(form, fused):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    world, d, n = 2, 128256 // 8 + 3, 2048
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, d, n, form, q, fused)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, same, arg, err in results:
        assert same, f"rank {rank}: gathered logits differ from the single-GPU GEMV"
        assert arg, f"rank {rank}: argmax differs"
        assert err == 0


def _ffn_full(dev, form, dim, hidden):
    """Weights of one Llama-3.2-1B FFN block, the same on every rank."""
    from minillama_infra_b200 import synth

    gate = synth.weights_gpu(hidden, dim, seed=301, device=dev)
    up = synth.weights_gpu(hidden, dim, seed=302, device=dev)
    down = synth.weights_gpu(dim, hidden, seed=303, device=dev)
    x = synth.activation_gpu(dim, 304, dev, outliers=(form == "w8a8"))
    return gate, up, down, x


def _ffn_single_gpu(gate, up, down, x, form, dim, hidden):
    from minillama_infra_b200.shard import ShardedFFN

    ffn = ShardedFFN(gate[0], gate[1], up[0], up[1], down[0], down[1], dim, hidden, 0, 1, form=form)
    xb = ffn.forward(x).clone()
    hb = ffn.hidden_vector().clone()
    torch.cuda.synchronize()
    ffn.close()
    return hb, xb


@pytest.mark.parametrize("form", ["w8a32", "w8a8"])
def test_ffn_block_one_gpu_matches_single_calls(form):
    """The FFN block (world 1) against single GEMV calls and the reference's
    elementwise silu_mul (src/model_cuda_v2_shared.cu:220-227) in fp32."""
    import numpy as np

    from minillama_infra_b200 import ops
    from oracle import oracle as orc

    dev = torch.device("cuda", 0)
    dim, hidden = 2048, 8192
    gate, up, down, x = _ffn_full(dev, form, dim, hidden)
    hb, xb = _ffn_single_gpu(gate, up, down, x, form, dim, hidden)

    def single(y, xv, w, n, d):
        if form == "w8a32":
            ops.matmul_int8(y, xv, w[0], w[1], n, d, 64)
        else:
            ops.matmul_dp4a_fused(y, xv, w[0], w[1], n, d, 64)

    g = torch.empty(hidden, device=dev)
    u = torch.empty(hidden, device=dev)
    single(g, x, gate, dim, hidden)
    single(u, x, up, dim, hidden)
    h_ref = (g * (1.0 / (1.0 + torch.exp(-g)))) * u
    xb_ref = torch.empty(dim, device=dev)
    single(xb_ref, hb, down, hidden, dim)  # down on the block's own hb: identical input
    torch.cuda.synchronize()
    assert orc.max_abs_rel(hb.cpu().numpy(), h_ref.cpu().numpy()) <= 1e-6
    assert np.array_equal(xb.cpu().numpy().view(np.uint32), xb_ref.cpu().numpy().view(np.uint32))
    assert ops.device_error() == 0


def _ffn_worker(rank, world, port, form, q):
    from datetime import timedelta

    import torch.distributed as dist

    from minillama_infra_b200 import ops
    from minillama_infra_b200.shard import ShardedFFN, row_shard

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    try:
        dim, hidden = 2048, 8192
        gate, up, down, x = _ffn_full(dev, form, dim, hidden)
        hb1, xb1 = _ffn_single_gpu(gate, up, down, x, form, dim, hidden)
        hs, ds = row_shard(hidden, world, rank), row_shard(dim, world, rank)
        ffn = ShardedFFN(gate[0][hs.r0:hs.r1].clone(), gate[1][hs.r0:hs.r1].clone(),
                         up[0][hs.r0:hs.r1].clone(), up[1][hs.r0:hs.r1].clone(),
                         down[0][ds.r0:ds.r1].clone(), down[1][ds.r0:ds.r1].clone(),
                         dim, hidden, rank, world, form=form)
        ok = True
        for _ in range(3):
            xb = ffn.forward(x)
            torch.cuda.synchronize()
            ok = ok and bool(torch.equal(xb.view(torch.int32), xb1.view(torch.int32)))
            ok = ok and bool(torch.equal(ffn.hidden_vector().view(torch.int32), hb1.view(torch.int32)))
        ffn.close()
        q.put((rank, ok, ops.device_error()))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("form", ["w8a32", "w8a8"])
def test_sharded_ffn_bit_exact_two_gpus(form):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ffn_worker, args=(r, world, port, form, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, ok, err in results:
        assert ok, f"rank {rank}: gathered hb / xb differ from the single-GPU block"
        assert err == 0


def _chain_ffn_worker(rank, world, port, form, q):
    """The fused FFN stack over `world` ranks (peer stores inside one chained
    launch per step) against the same stack on one GPU."""
    from datetime import timedelta

    import numpy as np
    import torch.distributed as dist

    from minillama_infra_b200 import ops, synth
    from minillama_infra_b200.shard import ChainShardedFFN, row_shard

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        dim, hidden, L = 2048, 8192, 4
        full = []
        for l in range(L):
            g = synth.weights_gpu(hidden, dim, seed=600 + 10 * l, device=dev)
            u = synth.weights_gpu(hidden, dim, seed=601 + 10 * l, device=dev)
            d = synth.weights_gpu(dim, hidden, seed=602 + 10 * l, device=dev)
            full.append((g[0], g[1], u[0], u[1], d[0], d[1]))
        x0 = synth.activation_gpu(dim, 699, dev, outliers=(form == "w8a8"))
        one = ChainShardedFFN(full, x0, dim, hidden, 0, 1, form=form)
        one.run()
        torch.cuda.synchronize()
        want = [one.hidden_rows(l)[0].view(np.uint32) for l in range(L)] + [one.output_rows()[0].view(np.uint32)]
        one.close()
        hs, ds = row_shard(hidden, world, rank), row_shard(dim, world, rank)
        mine = [(gq[hs.r0:hs.r1].clone(), gs[hs.r0:hs.r1].clone(), uq[hs.r0:hs.r1].clone(), us[hs.r0:hs.r1].clone(),
                 dq[ds.r0:ds.r1].clone(), dss[ds.r0:ds.r1].clone()) for (gq, gs, uq, us, dq, dss) in full]

        def exchange(h):
            out = [None] * world
            dist.all_gather_object(out, h)
            return out

        sh = ChainShardedFFN(mine, x0, dim, hidden, rank, world, form=form, exchange=exchange)
        dist.barrier()
        ok = True
        for rep in range(5):  # both mirror halves, several times
            sh.run()
            torch.cuda.synchronize()
            dist.barrier()  # every rank's rows of this run have landed everywhere
            got = [sh.hidden_rows(l) for l in range(L)] + [sh.output_rows()]
            for (v, tagged), w in zip(got, want):
                ok = ok and tagged and bool(np.array_equal(v.view(np.uint32), w))
            dist.barrier()
        err = ops.device_error()
        sh.close()
        q.put((rank, ok, err))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("form", ["w8a32", "w8a8"])
def test_chain_sharded_ffn_bit_exact_two_gpus(form):
    """Four FFN blocks row-sharded over two GPUs in one chained launch per
    step, the hb and x' rows exchanged by tagged peer stores inside the
    kernel: every layer's hb and the last x' are bit-identical to one GPU on
    both ranks, in five runs in a row."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_chain_ffn_worker, args=(r, world, port, form, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, ok, err in results:
        assert ok, f"rank {rank}: sharded chain rows differ from one GPU (or were not tagged)"
        assert err == 0
