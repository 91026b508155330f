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
