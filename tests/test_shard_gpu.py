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
            for step in range(5):  # both logits halves, several times
                out = lin.forward(x)
                torch.cuda.synchronize()
                got = torch.empty(d, dtype=torch.float32, device=dev)
                ops.copy_from_ptr(got, lin.logits(step & 1), d * 4)
                same = same and bool(torch.equal(got.view(torch.int32), full.view(torch.int32)))
                arg = arg and int(out.item()) == want
            lin.close()
        q.put((rank, same, arg, ops.device_error()))
        dist.barrier()
    finally:
        dist.destroy_process_group()


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
