"""CPU checks of the batch-1 GEMV launch planner (no GPU needed): every shape
of the Llama-3.2 1B / 3B decode and the classifier gets a plan that fits the
B200's shared memory with room for the next kernel's CTA, keeps the stage
ring at least double-buffered and covers every row exactly once."""
import ctypes

import pytest

from minillama_infra_b200 import _lib, synth

B200 = dict(sm_count=148, smem_per_sm=233472, smem_optin=232448)
FORMS = {"w8a32": 0, "w8a8": 1, "w8a8_fused": 2}
SHAPES = sorted({(d, n) for _, d, n in synth.LLAMA_1B + synth.LLAMA_3B} | {synth.CLASSIFIER_1B[1:]}
                | {(16032, 2048), (64128, 2048), (1, 256), (37, 1280), (5, 16384)})


def plan(form, n, d, dev=B200):
    out = (ctypes.c_int * 8)()
    rc = _lib.lib().mli_debug_plan_gemv(FORMS[form], n, d, dev["sm_count"], dev["smem_per_sm"],
                                        dev["smem_optin"], out)
    return rc, dict(zip(["grid", "smem", "S", "wps", "R", "stages", "ring", "stage_bytes"], out))


@pytest.mark.parametrize("form", list(FORMS))
@pytest.mark.parametrize("d,n", SHAPES)
def test_plan_fits_and_covers(form, d, n):
    rc, p = plan(form, n, d)
    if form == "w8a32" and n > 8192:
        assert rc == _lib.MLI_ERR_UNSUPPORTED  # more than eight 1024-column slices
        return
    assert rc == _lib.MLI_OK
    assert 1 <= p["grid"] <= 2 * B200["sm_count"]
    if p["stages"] < 2 * B200["sm_count"]:
        assert p["grid"] <= B200["sm_count"]  # leaves room for the next kernel
    assert p["grid"] <= p["stages"]
    assert p["stages"] * p["R"] >= d > (p["stages"] - 1) * p["R"]
    assert 2 <= p["ring"] <= 6
    assert p["S"] * p["wps"] <= 8 and p["R"] % p["wps"] == 0
    slice_cols = 1024 if form == "w8a32" else 2048
    assert p["S"] == -(-n // slice_cols)
    assert p["stage_bytes"] == p["R"] * n + p["R"] * (n // 64) * 4
    assert p["stage_bytes"] % 16 == 0
    # two CTAs (this kernel and the next one in the stream) fit on one SM
    if n <= 8192:
        assert 2 * (p["smem"] + 1024) <= B200["smem_per_sm"]
    assert p["smem"] <= B200["smem_optin"]


def test_plan_rejects_bad_arguments():
    out = (ctypes.c_int * 8)()
    l = _lib.lib()
    assert l.mli_debug_plan_gemv(3, 2048, 2048, 148, 233472, 232448, out) == _lib.MLI_ERR_INVALID_ARG
    assert l.mli_debug_plan_gemv(0, 2048, 0, 148, 233472, 232448, out) == _lib.MLI_ERR_INVALID_ARG
    assert l.mli_debug_plan_gemv(0, 2000, 64, 148, 233472, 232448, out) == _lib.MLI_ERR_UNSUPPORTED


# ---------------------------------------------------------------------------
# Chain planner (mli_debug_plan_chain): fake, aligned device addresses only.
# ---------------------------------------------------------------------------
def _chain(layers=16, form=0, n_x=None):
    """Decode-structured chain of the Llama-3.2-1B layer GEMVs."""
    from minillama_infra_b200.ops import DECODE_LAYER_WAITS

    mb = 1 << 20
    arr = (_lib.GemvOp * (7 * layers))()
    # activation buffers: 1 = layer input (q/k/v), 2 = attention out (o),
    # 3 = ffn input (gate/up), 4 = SwiGLU out (down); reused by every layer
    src = [1, 1, 1, 2, 3, 3, 4]
    for l in range(layers):
        for i, (_, d, n) in enumerate(synth.LLAMA_1B):
            e = arr[7 * l + i]
            e.form, e.n, e.d, e.group_size = form, n, d, 64
            e.wait = 7 * l + DECODE_LAYER_WAITS[i]
            if form == 1:
                e.xq, e.xs = mb * (10 + src[i]), mb * (20 + src[i])
            else:
                e.x = mb * (10 + src[i])
            e.y = mb * (100 + 7 * l + i)
            e.w_q, e.w_s = mb * (1000 + 7 * l + i), mb * (2000 + 7 * l + i)
    return arr


def plan_chain(arr, count=None, sm=148, optin=232448):
    out = (ctypes.c_int * 7)()
    rc = _lib.lib().mli_debug_plan_chain(arr, len(arr) if count is None else count, sm, optin, out)
    return rc, dict(zip(["grid", "smem", "ring", "slot", "units", "epochs", "phases"], out))


@pytest.mark.parametrize("form", [0, 1, 2])
def test_chain_plan_llama_step(form):
    arr = _chain(16, form)
    rc, p = plan_chain(arr)
    assert rc == _lib.MLI_OK
    assert p["grid"] == 148
    assert p["smem"] <= B200["smem_optin"]
    assert 2 <= p["ring"] <= 6
    # every op's stage is 64 row slices of 1024 columns (W8A32) or 32 of 2048
    # (W8A8): 64 KB of weights plus their scales, whatever n is
    assert p["slot"] == 65536 + 65536 // 64 * 4
    units = 0
    for _, d, n in synth.LLAMA_1B:
        rows = 65536 // n  # rows per stage
        units += -(-d // rows)
    assert p["units"] == 16 * units
    # q/k/v share the layer input, gate/up the ffn input: 4 activations a layer
    assert p["epochs"] == 16 * 4
    # q/k/v, o, gate/up, down: 4 dependency phases a layer
    assert p["phases"] == 16 * 4


def test_chain_plan_rejects_bad_chains():
    arr = _chain(1)
    assert plan_chain(arr)[0] == _lib.MLI_OK
    bad = _chain(1)
    bad[3].wait = 4  # waits for itself
    assert plan_chain(bad)[0] == _lib.MLI_ERR_INVALID_ARG
    bad = _chain(1)
    bad[2].form = 2  # mixed forms
    assert plan_chain(bad)[0] == _lib.MLI_ERR_INVALID_ARG
    bad = _chain(1)
    bad[1].y = bad[1].x  # output over its own activation
    assert plan_chain(bad)[0] == _lib.MLI_ERR_INVALID_ARG
    bad = _chain(1)
    bad[0].w_q = None
    assert plan_chain(bad)[0] == _lib.MLI_ERR_INVALID_ARG
    bad = _chain(1)
    bad[4].n = 2000  # not a multiple of 256
    assert plan_chain(bad)[0] == _lib.MLI_ERR_UNSUPPORTED
    bad = _chain(1)
    bad[5].group_size = 32
    assert plan_chain(bad)[0] == _lib.MLI_ERR_UNSUPPORTED
    bad = _chain(1)
    bad[5].w_s += 4  # misaligned scales
    assert plan_chain(bad)[0] == _lib.MLI_ERR_UNSUPPORTED
    assert plan_chain(arr, count=0)[0] == _lib.MLI_ERR_INVALID_ARG
    out = (ctypes.c_int * 7)()
    assert _lib.lib().mli_debug_plan_chain(None, 3, 148, 232448, out) == _lib.MLI_ERR_INVALID_ARG
    # W8A32 rows wider than eight 1024-column slices do not fit the row kernels
    wide = _chain(1)
    wide[6].n = 16384
    assert plan_chain(wide)[0] == _lib.MLI_ERR_UNSUPPORTED


def test_chain_plan_independent_ops_form_one_phase():
    arr = _chain(2)
    for e in arr:
        e.wait = 0
    rc, p = plan_chain(arr)
    assert rc == _lib.MLI_OK and p["phases"] == 1


def _ffn_chain(form=0):
    """gate (SwiGLU with the next op), up (its companion), down (add into the residual)."""
    mb = 1 << 20
    arr = (_lib.GemvOp * 3)()
    for i, (d, n) in enumerate([(8192, 2048), (8192, 2048), (2048, 8192)]):
        e = arr[i]
        e.form, e.n, e.d, e.group_size = form, n, d, 64
        e.w_q, e.w_s = mb * (100 + i), mb * (200 + i)
    arr[0].x = arr[1].x = mb * 10
    arr[0].y = mb * 20            # h
    arr[0].epilogue = 2
    arr[1].y = None               # the companion's output is unused
    arr[2].x, arr[2].y, arr[2].wait, arr[2].epilogue = mb * 20, mb * 30, 2, 1
    return arr


@pytest.mark.parametrize("form", [0, 2])
def test_chain_plan_swiglu_pair_and_add(form):
    rc, p = plan_chain(_ffn_chain(form))
    assert rc == _lib.MLI_OK
    # a SwiGLU stage holds half the rows of a plain one (gate + up rows together);
    # the companion adds no units
    rows_gate = 65536 // 2048 // 2
    rows_down = 65536 // 8192
    assert p["units"] == -(-8192 // rows_gate) + -(-2048 // rows_down)
    assert p["phases"] == 2


def test_chain_plan_rejects_bad_epilogues():
    bad = _ffn_chain()
    bad[1].n = 4096               # companion shape differs from its gate
    assert plan_chain(bad)[0] == _lib.MLI_ERR_INVALID_ARG
    bad = _ffn_chain()
    bad[1].wait = 1               # companion waits differently
    assert plan_chain(bad)[0] == _lib.MLI_ERR_INVALID_ARG
    bad = _ffn_chain()
    bad[1].epilogue = 1           # companion with its own epilogue
    assert plan_chain(bad)[0] == _lib.MLI_ERR_INVALID_ARG
    bad = _ffn_chain()
    bad[2].epilogue = 2           # SwiGLU on the last op: no companion
    assert plan_chain(bad)[0] == _lib.MLI_ERR_INVALID_ARG
    bad = _ffn_chain()
    bad[2].epilogue = 5
    assert plan_chain(bad)[0] == _lib.MLI_ERR_INVALID_ARG
    bad = _ffn_chain()
    bad[0].y = None               # the gate's output is required
    assert plan_chain(bad)[0] == _lib.MLI_ERR_INVALID_ARG
