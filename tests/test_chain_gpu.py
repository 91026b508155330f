"""GPU checks of the chained GEMV launch (mli_chain_*) through the C ABI.

Every op of a chain must give exactly (bit for bit) the output of its single
call -- matmul_int8 / matmul_dp4a / matmul_dp4a_fused, whose own parity with
the oracle is covered by test_gpu_parity.py -- whatever the dependencies:
independent ops, a pure dependency chain (x of op i = y of op i - 1), and the
decode structure with activation buffers reused by every layer (which also
checks that no SM reads a stale activation from its L1).  One op of each
chain is also checked against the oracle directly.
"""
import numpy as np
import pytest

from oracle import oracle as orc
from minillama_infra_b200 import ops, synth
from minillama_infra_b200._lib import MliError, lib

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu
TOL = {"w8a32": 1e-5, "w8a8": 1e-6, "w8a8_fused": 1e-6}


def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda:0")


def weights(d, n, seed):
    return synth.weights_gpu(d, n, seed=seed, device=dev())


def single(form, y, x, q, s, n, d, xq=None, xs=None):
    if form == "w8a32":
        ops.matmul_int8(y, x, q, s, n, d, 64)
    elif form == "w8a8":
        ops.matmul_dp4a(y, xq, xs, q, s, n, d, 64)
    else:
        ops.matmul_dp4a_fused(y, x, q, s, n, d, 64)


def bits(t):
    return t.cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("form", ["w8a32", "w8a8", "w8a8_fused"])
def test_chain_independent_ops_match_single_calls(form):
    shapes = [(2048, 2048), (512, 2048), (512, 2048), (2048, 2048), (8192, 2048), (8192, 2048),
              (2048, 8192), (300, 512), (37, 3072), (5, 1280)]
    chain, refs = [], []
    for i, (d, n) in enumerate(shapes):
        q, s = weights(d, n, 50 + i)
        x = torch.from_numpy(synth.activation_np(n, 90 + i, outliers=form != "w8a32")).to(dev())
        op = dict(form=form, n=n, d=d, wait=0, w_q=q, w_s=s, y=torch.full((d,), float("nan"), device=dev()))
        ref = torch.empty(d, device=dev())
        if form == "w8a8":
            xq = torch.empty(n, dtype=torch.int8, device=dev())
            xs = torch.empty(1, device=dev())
            ops.quantize_activation(xq, xs, x, n)
            op.update(xq=xq, xs=xs)
            single(form, ref, None, q, s, n, d, xq, xs)
        else:
            op.update(x=x)
            single(form, ref, x, q, s, n, d)
        chain.append(op)
        refs.append(ref)
    c = ops.GemvChain(chain)
    for rep in range(3):  # counters return to zero between runs
        for op in chain:
            op["y"].fill_(float("nan"))
        c.run()
        torch.cuda.synchronize()
        for i, (op, ref) in enumerate(zip(chain, refs)):
            assert np.array_equal(bits(op["y"]), bits(ref)), (rep, i, shapes[i])
    c.close()
    assert ops.device_error() == 0


@pytest.mark.parametrize("form", ["w8a32", "w8a8_fused"])
def test_chain_dependencies_match_sequential_calls(form):
    """x of op i is y of op i - 1 (wait = i): every op needs the whole output
    of the previous one, produced by other SMs in the same launch."""
    dims = [2048, 8192, 2048, 2048, 512, 1024, 8192, 2048]
    bufs = [torch.from_numpy(synth.activation_np(dims[0], 7)).to(dev())]
    bufs += [torch.full((d,), float("nan"), device=dev()) for d in dims[1:]]
    ws = [weights(dims[i + 1], dims[i], 300 + i) for i in range(len(dims) - 1)]
    chain = [dict(form=form, n=dims[i], d=dims[i + 1], wait=i, x=bufs[i], y=bufs[i + 1],
                  w_q=ws[i][0], w_s=ws[i][1]) for i in range(len(dims) - 1)]
    # sequential single calls into separate buffers
    seq = [bufs[0].clone()] + [torch.empty(d, device=dev()) for d in dims[1:]]
    for i in range(len(dims) - 1):
        single(form, seq[i + 1], seq[i], ws[i][0], ws[i][1], dims[i], dims[i + 1])
    torch.cuda.synchronize()
    c = ops.GemvChain(chain)
    for rep in range(3):
        for b in bufs[1:]:
            b.fill_(float("nan"))
        c.run()
        torch.cuda.synchronize()
        for i in range(1, len(dims)):
            assert np.array_equal(bits(bufs[i]), bits(seq[i])), (rep, i)
    # first op against the oracle
    x0 = bufs[0].cpu().numpy()
    wq, wsc = ws[0][0].cpu().numpy(), ws[0][1].cpu().numpy()
    if form == "w8a32":
        ref = orc.gemv_w8a32_f64(x0, wq, wsc)
    else:
        xq, xs = orc.quantize_activation(x0)
        ref = orc.gemv_w8a8_f64(xq, xs, wq, wsc)
    assert orc.max_abs_rel(bufs[1].cpu().numpy(), ref) <= TOL[form]
    c.close()
    assert ops.device_error() == 0


def _decode_chain(form, layers):
    """Llama-3.2-1B layer GEMVs in decode order with the decode waits.  Four
    activation buffers are reused by every layer, as in a forward pass: q/k/v
    read A (the previous layer's down output), o reads q's output (standing in
    for attention), gate/up read o's output, down reads gate's output."""
    A = torch.from_numpy(synth.activation_np(2048, 11)).to(dev())
    Q = torch.empty(2048, device=dev())
    K = torch.empty(512, device=dev())
    V = torch.empty(512, device=dev())
    O = torch.empty(2048, device=dev())
    Gt = torch.empty(8192, device=dev())
    U = torch.empty(8192, device=dev())
    outs = {"q": Q, "k": K, "v": V, "o": O, "gate": Gt, "up": U}
    srcs = {"q": A, "k": A, "v": A, "o": Q, "gate": O, "up": O, "down": Gt}
    w = [[weights(d, n, 1000 * l + i) for i, (_, d, n) in enumerate(synth.LLAMA_1B)] for l in range(layers)]
    names = ["q", "k", "v", "o", "gate", "up", "down"]
    chain = []
    for l in range(layers):
        for i, (_, d, n) in enumerate(synth.LLAMA_1B):
            nm = names[i]
            chain.append(dict(form=form, n=n, d=d, wait=7 * l + ops.DECODE_LAYER_WAITS[i],
                              x=srcs[nm], y=outs.get(nm, A), w_q=w[l][i][0], w_s=w[l][i][1]))
    return A, outs, w, chain


@pytest.mark.parametrize("form", ["w8a32", "w8a8_fused"])
def test_chain_decode_structure_reused_buffers(form):
    layers = 3
    A, outs, w, chain = _decode_chain(form, layers)
    a0 = A.clone()
    # reference: the same calls one by one (every layer feeds the next, so the
    # final buffers depend on every op)
    for l in range(layers):
        for i, (_, d, n) in enumerate(synth.LLAMA_1B):
            op = chain[7 * l + i]
            single(form, op["y"], op["x"], op["w_q"], op["w_s"], n, d)
    torch.cuda.synchronize()
    final = {k: bits(v) for k, v in outs.items()}
    final["a"] = bits(A)
    c = ops.GemvChain(chain)
    for rep in range(2):
        A.copy_(a0)
        for t in outs.values():
            t.fill_(float("nan"))
        c.run()
        torch.cuda.synchronize()
        assert np.array_equal(bits(A), final["a"]), rep
        for k, t in outs.items():
            assert np.array_equal(bits(t), final[k]), (rep, k)
    # the same chain captured into a CUDA graph and replayed
    stream = torch.cuda.Stream()
    A.copy_(a0)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        c.run()
    for rep in range(2):
        A.copy_(a0)
        g.replay()
        torch.cuda.synchronize()
        assert np.array_equal(bits(A), final["a"]), ("graph", rep)
        assert np.array_equal(bits(outs["up"]), final["up"]), ("graph", rep)
    del g
    c.close()
    assert ops.device_error() == 0


def test_chain_rejects_bad_arguments():
    l = lib()
    assert l.mli_chain_run(None, None) == 1
    assert l.mli_chain_destroy(None) == 1
    q, s = weights(64, 256, 1)
    x = torch.zeros(256, device=dev())
    y = torch.zeros(64, device=dev())
    with pytest.raises(MliError):
        ops.GemvChain([dict(form="w8a32", n=256, d=64, wait=1, x=x, y=y, w_q=q, w_s=s)])
    with pytest.raises(MliError):
        ops.GemvChain([dict(form="w8a32", n=192, d=64, wait=0, x=x, y=y, w_q=q, w_s=s)])


@pytest.mark.parametrize("form", ["w8a32", "w8a8_fused"])
def test_chain_swiglu_and_residual_epilogues(form):
    """One chain: h = silu(W1 x) * (W3 x) (SwiGLU pair), then res += W2 h.
    Against single calls followed by the reference's elementwise steps
    (silu_mul, add: src/model_cuda_v2_shared.cu:215-227) in fp32."""
    dim, hidden = 2048, 8192
    w1 = weights(hidden, dim, 71)
    w3 = weights(hidden, dim, 72)
    w2 = weights(dim, hidden, 73)
    x = torch.from_numpy(synth.activation_np(dim, 74, outliers=form != "w8a32")).to(dev())
    res0 = torch.from_numpy(synth.activation_np(dim, 75)).to(dev())
    g = torch.empty(hidden, device=dev())
    u = torch.empty(hidden, device=dev())
    single(form, g, x, w1[0], w1[1], dim, hidden)
    single(form, u, x, w3[0], w3[1], dim, hidden)
    h_ref = g * (1.0 / (1.0 + torch.exp(-g)))
    h_ref = h_ref * u
    v = torch.empty(dim, device=dev())
    single(form, v, h_ref, w2[0], w2[1], hidden, dim)
    res_ref = res0 + v
    torch.cuda.synchronize()

    h = torch.full((hidden,), float("nan"), device=dev())
    res = res0.clone()
    c = ops.GemvChain([
        dict(form=form, n=dim, d=hidden, wait=0, x=x, y=h, w_q=w1[0], w_s=w1[1], epilogue="swiglu"),
        dict(form=form, n=dim, d=hidden, wait=0, x=x, y=None, w_q=w3[0], w_s=w3[1]),
        dict(form=form, n=hidden, d=dim, wait=2, x=h, y=res, w_q=w2[0], w_s=w2[1], epilogue="add"),
    ])
    for rep in range(2):
        res.copy_(res0)
        h.fill_(float("nan"))
        c.run()
        torch.cuda.synchronize()
        hn, hr = h.cpu().numpy(), h_ref.cpu().numpy()
        assert not np.isnan(hn).any()
        assert orc.max_abs_rel(hn, hr) <= 1e-6, rep
        assert orc.max_abs_rel(res.cpu().numpy(), res_ref.cpu().numpy()) <= 1e-5, rep
    c.close()
    assert ops.device_error() == 0


def _norm_weights(n, seed):
    rng = np.random.default_rng(seed)
    return (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)


@pytest.mark.parametrize("form", ["w8a32", "w8a8_fused"])
def test_chain_decode_layers_with_norm_prologue(form):
    """Two Llama-3.2-1B decode layers as one chain, with everything of the
    layer but attention: q/k/v read RMSNorm(resid) (the norm in the op's
    prologue, src/model_cuda_v2_shared.cu:381), o reads q's output (standing
    in for attention) and adds into resid (:402-405), gate/up read
    RMSNorm(resid) as one SwiGLU pair (:405-410), down adds into resid
    (:412-414).  Every activation is another op's output of the same launch,
    handed over through the tagged mirrors.  Checked step by step against
    single calls on the oracle's RMSNorm (restated in the prologue's sum
    order): q/k/v, o, down and the final residual bit for bit, the SwiGLU
    product within 1e-6 (expf)."""
    layers, dim, hidden = 2, 2048, 8192
    resid0 = synth.activation_np(dim, 500)
    resid = torch.from_numpy(resid0.copy()).to(dev())
    att_w = [_norm_weights(dim, 600 + l) for l in range(layers)]
    ffn_w = [_norm_weights(dim, 700 + l) for l in range(layers)]
    t_att = [torch.from_numpy(a).to(dev()) for a in att_w]
    t_ffn = [torch.from_numpy(a).to(dev()) for a in ffn_w]
    w = [[weights(d, n, 2000 * l + i) for i, (_, d, n) in enumerate(synth.LLAMA_1B)] for l in range(layers)]
    bufs = [{nm: torch.full((d,), float("nan"), device=dev()) for nm, d in
             (("q", dim), ("k", 512), ("v", 512), ("h", hidden))} for _ in range(layers)]
    chain = []
    for l in range(layers):
        b, W, B = 7 * l, w[l], bufs[l]
        chain += [
            dict(form=form, n=dim, d=dim, wait=b, x=resid, norm_w=t_att[l], y=B["q"], w_q=W[0][0], w_s=W[0][1]),
            dict(form=form, n=dim, d=512, wait=b, x=resid, norm_w=t_att[l], y=B["k"], w_q=W[1][0], w_s=W[1][1]),
            dict(form=form, n=dim, d=512, wait=b, x=resid, norm_w=t_att[l], y=B["v"], w_q=W[2][0], w_s=W[2][1]),
            dict(form=form, n=dim, d=dim, wait=b + 3, x=B["q"], y=resid, epilogue="add", w_q=W[3][0],
                 w_s=W[3][1]),
            dict(form=form, n=dim, d=hidden, wait=b + 4, x=resid, norm_w=t_ffn[l], y=B["h"], epilogue="swiglu",
                 w_q=W[4][0], w_s=W[4][1]),
            dict(form=form, n=dim, d=hidden, wait=b + 4, x=resid, norm_w=t_ffn[l], y=None, w_q=W[5][0],
                 w_s=W[5][1]),
            dict(form=form, n=hidden, d=dim, wait=b + 6, x=B["h"], y=resid, epilogue="add", w_q=W[6][0],
                 w_s=W[6][1]),
        ]
    c = ops.GemvChain(chain)
    for rep in range(3):  # the launch sequence advances: later runs must not take old rows
        resid.copy_(torch.from_numpy(resid0))
        for B in bufs:
            for t in B.values():
                t.fill_(float("nan"))
        c.run()
        torch.cuda.synchronize()
        exp = resid0.copy()
        for l in range(layers):
            W, B = w[l], bufs[l]

            def one(x_np, i, d, n):
                y = torch.empty(d, device=dev())
                single(form, y, torch.from_numpy(np.ascontiguousarray(x_np, np.float32)).to(dev()),
                       W[i][0], W[i][1], n, d)
                return y.cpu().numpy()

            xa = orc.rmsnorm_chain(exp, att_w[l])
            for i, nm in ((0, "q"), (1, "k"), (2, "v")):
                got = B[nm].cpu().numpy()
                assert np.array_equal(got.view(np.uint32), one(xa, i, got.size, dim).view(np.uint32)), (rep, l, nm)
            exp = (exp + one(B["q"].cpu().numpy(), 3, dim, dim)).astype(np.float32)
            xf = orc.rmsnorm_chain(exp, ffn_w[l])
            g = torch.from_numpy(one(xf, 4, hidden, dim))
            u = torch.from_numpy(one(xf, 5, hidden, dim))
            h_ref = ((g * (1.0 / (1.0 + torch.exp(-g)))) * u).numpy()
            h = B["h"].cpu().numpy()
            assert not np.isnan(h).any()
            assert orc.max_abs_rel(h, h_ref) <= 1e-6, (rep, l)
            exp = (exp + one(h, 6, dim, hidden)).astype(np.float32)
        assert np.array_equal(resid.cpu().numpy().view(np.uint32), exp.view(np.uint32)), rep
    c.close()
    assert ops.device_error() == 0


def test_chain_rejects_reading_an_unawaited_producer():
    """An op reading an earlier op's output must wait for it."""
    q, s = weights(256, 256, 1)
    x = torch.zeros(256, device=dev())
    y = torch.zeros(256, device=dev())
    z = torch.zeros(256, device=dev())
    with pytest.raises(MliError):
        ops.GemvChain([dict(form="w8a32", n=256, d=256, wait=0, x=x, y=y, w_q=q, w_s=s),
                       dict(form="w8a32", n=256, d=256, wait=0, x=y, y=z, w_q=q, w_s=s)])


def _ffn_layers(dim, hidden, layers, seed):
    out = []
    for l in range(layers):
        g = weights(hidden, dim, seed + 10 * l)
        u = weights(hidden, dim, seed + 10 * l + 1)
        d = weights(dim, hidden, seed + 10 * l + 2)
        out.append((g[0], g[1], u[0], u[1], d[0], d[1]))
    return out


@pytest.mark.parametrize("form", ["w8a32", "w8a8"])
def test_sharded_chain_one_rank_matches_plain_chain(form):
    """A row-sharded FFN stack (mli_chain_create_sharded) on one rank gives
    the plain chain's hb and x' bit for bit, read back from its mirrors with
    every row tagged, over several runs (both mirror halves in turn)."""
    from minillama_infra_b200.shard import ChainShardedFFN

    dim, hidden, L = 2048, 8192, 3
    layers = _ffn_layers(dim, hidden, L, 500)
    x0 = torch.from_numpy(synth.activation_np(dim, 77, outliers=form == "w8a8")).to(dev())
    f = "w8a32" if form == "w8a32" else "w8a8_fused"
    hb = torch.zeros(hidden, device=dev())
    xb = torch.zeros(dim, device=dev())
    plain_ops = []
    for l, (gq, gs, uq, us, dq, ds_) in enumerate(layers):
        x = x0 if l == 0 else xb
        plain_ops += [dict(form=f, n=dim, d=hidden, wait=3 * l, x=x, y=hb, w_q=gq, w_s=gs, epilogue="swiglu"),
                      dict(form=f, n=dim, d=hidden, wait=3 * l, x=x, y=None, w_q=uq, w_s=us),
                      dict(form=f, n=hidden, d=dim, wait=3 * l + 2, x=hb, y=xb, w_q=dq, w_s=ds_)]
    plain = ops.GemvChain(plain_ops)
    plain.run()
    torch.cuda.synchronize()
    want_h, want_x = bits(hb), bits(xb)
    sh = ChainShardedFFN(layers, x0, dim, hidden, 0, 1, form=form)
    for rep in range(3):
        sh.run()
        torch.cuda.synchronize()
        h, h_ok = sh.hidden_rows(L - 1)
        x, x_ok = sh.output_rows()
        assert h_ok and x_ok, rep
        assert np.array_equal(h.view(np.uint32), want_h), rep
        assert np.array_equal(x.view(np.uint32), want_x), rep
        assert np.array_equal(bits(sh.xb[:dim]), want_x), rep  # the rank's own rows in its y
    sh.close()
    plain.close()
    assert ops.device_error() == 0


def test_sharded_chain_times_out_when_a_rank_never_delivers():
    """Rank 0 of a two-rank FFN layer whose partner never runs: its rows of hb
    never arrive, so the down projection's bounded wait runs out -- the launch
    ends with device error 4 instead of hanging, and the GPU stays usable.
    The partner's mirror is stood in for by a zeroed buffer of this GPU.
    Running before the peers are set is refused."""
    from minillama_infra_b200.shard import ChainShardedFFN, row_shard

    dim, hidden = 2048, 8192
    (gq, gs, uq, us, dq, ds_), = _ffn_layers(dim, hidden, 1, 800)
    hs, dsh = row_shard(hidden, 2, 0), row_shard(dim, 2, 0)
    mine = [(gq[hs.r0:hs.r1].clone(), gs[hs.r0:hs.r1].clone(), uq[hs.r0:hs.r1].clone(), us[hs.r0:hs.r1].clone(),
             dq[dsh.r0:dsh.r1].clone(), ds_[dsh.r0:dsh.r1].clone())]
    x0 = torch.from_numpy(synth.activation_np(dim, 81)).to(dev())
    sh = ChainShardedFFN(mine, x0, dim, hidden, 0, 2, form="w8a32")
    with pytest.raises(MliError):
        sh.run()  # no peers yet
    assert ops.device_error() == 0
    partner = torch.zeros(8 << 20, dtype=torch.uint8, device=dev())  # larger than the mirror block
    sh.chain.set_peer_pointers([0, partner.data_ptr()], 0)
    sh.run()
    torch.cuda.synchronize()
    assert ops.device_error() == 4
    _, complete = sh.output_rows()
    assert not complete
    sh.close()
    y = torch.empty(64, device=dev())  # the context still works
    ops.matmul_int8(y, x0, gq[:64].contiguous(), gs[:64].contiguous(), dim, 64, 64)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
