"""Decision inputs on the GPU: IRAP importance (compute_irap_importance, the agent's contract
wrappers) and decide_reuse_per_token, against the reference fixtures and the CPU oracle.

Tolerances are the reference's own: importance within 1e-6 (its vectorised-vs-scalar golden
tests), the EMA within 1e-6 relative, delta_a within 1e-5 relative.  The reuse mask must equal
the reference's except where the reference's float32 drift lies within 1e-6 (relative) of
its threshold.  Against the oracle (float64 reductions) the drift agrees to 4 ulp and the mask
exactly away from the threshold; importance agrees within 1e-6 except for tokens whose EMA is
within a few ulp of another token's in the same head (their ranks may swap, one rank step).
"""

import numpy as np
import pytest
import torch

from golden_lib import case_arrays, irap_scores, load_pins, reuse_inputs
from oracle import decision_oracle as DO

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def skv():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import shadow_infer_b200.shadowkv as m
    return m


def _cases(kind):
    return sorted(c for c, v in load_pins()["cases"].items() if v["kind"] == kind)


def _agent():
    from shadow_infer_b200.shadowkv.shadowkv_agent import ShadowKVAgent
    return ShadowKVAgent({"num_layers": 4, "num_heads": 8, "head_dim": 64})


@pytest.mark.parametrize("case", _cases("reuse_decision"))
def test_reuse_decision_matches_reference_fixture(case, skv, golden_small):
    from shadow_infer_b200.shadowkv.shadowkv_agent import decide_reuse_mask
    pin = load_pins()["cases"][case]
    a = case_arrays(golden_small, case)
    k, v, kp, vp, imp = (torch.from_numpy(x).cuda() for x in reuse_inputs(pin["seed"], pin["B"], pin["H"], pin["S"],
                                                                           pin["D"]))
    mask, stats, drift = decide_reuse_mask(k, v, kp, vp, pin["step_id"], pin["total_steps"], pin["drift"],
                                           pin["mode"], imp, return_drift=True)
    np.testing.assert_allclose(drift.cpu().numpy().astype(np.float64), a["ref_delta"], rtol=1e-6, atol=0)
    near = np.abs(a["ref_delta"] - a["ref_thr"]) <= 1e-6 * a["ref_thr"]
    got = mask.cpu().numpy()
    assert np.array_equal(got[~near], a["mask"].astype(bool)[~near])
    if not near.any():
        assert stats == pin["stats"]
    # the agent method returns the reference's dict
    d, st2 = _agent().decide_reuse_per_token(k, v, kp, vp, pin["step_id"], pin["total_steps"], pin["drift"],
                                              pin["mode"], imp)
    assert st2 == stats and len(d) == pin["S"] * pin["H"]
    assert all(d[(t, h)] == bool(got[t, h]) for t in range(pin["S"]) for h in range(pin["H"]))


@pytest.mark.parametrize("B,H,S,D,step,total,drift,mode", [
    (1, 32, 1024, 128, 4, 16, 0.3, "balanced"),
    (2, 16, 777, 64, 0, 8, 0.0, "aggressive"),
    (3, 8, 300, 96, 7, 8, 0.6, "conservative"),
    (1, 4, 129, 30, 2, 4, 0.1, "balanced"),        # head_dim not a multiple of 4: scalar loads
])
def test_reuse_decision_matches_oracle(skv, B, H, S, D, step, total, drift, mode):
    from shadow_infer_b200.shadowkv.shadowkv_agent import decide_reuse_mask
    k, v, kp, vp, imp = reuse_inputs(S * 13 + D, B, H, S, D)
    imp[5, 0] = np.nan                               # NaN importance: threshold NaN, never reused
    om, ostats, odrift = DO.decide_reuse_per_token(k, v, kp, vp, step, total, drift, mode, imp)
    t = [torch.from_numpy(x).cuda() for x in (k, v, kp, vp, imp)]
    mask, stats, gdrift = decide_reuse_mask(*t[:4], step, total, drift, mode, t[4], return_drift=True)
    # float32 partials of four squares each (< 2^-22 relative), then the reference's float32
    # ratio steps: a few ulp from the oracle's float64 sums, far inside the 1e-6 threshold band
    np.testing.assert_array_max_ulp(gdrift.cpu().numpy(), odrift.T, maxulp=4)
    eff = DO.effective_threshold(step, total, drift, mode)
    thr = np.maximum(eff * (1.0 - 0.3 * np.clip(imp.astype(np.float64), 0.0, 1.0)), 1e-5)
    near = np.abs(odrift.T.astype(np.float64) - thr) <= 1e-6 * thr
    got = mask.cpu().numpy()
    assert np.array_equal(got[~near], om[~near])
    if not near.any():
        assert stats == ostats
    assert not bool(mask[5, 0])


def _irap_inputs(pin, a):
    x = irap_scores(pin["seed"], pin["B"], pin["H"], pin["Sq"], pin["Sk"], kind=pin["score_kind"], bad=pin["bad"])
    prev = a.get("prev")
    return x, prev


@pytest.mark.parametrize("case", _cases("irap"))
def test_irap_matches_reference_fixture(case, skv, golden_small):
    pin = load_pins()["cases"][case]
    a = case_arrays(golden_small, case)
    x, prev = _irap_inputs(pin, a)
    xt = torch.from_numpy(x).cuda()
    pt = None if prev is None else torch.from_numpy(prev).cuda()
    if pin["contract"] is None:
        imp, ema, da = skv.compute_irap_importance(xt, pt, pin["decay"], pin["beta"], pin["sink"], pin["layer_index"],
                                                   pin["num_layers"])
    else:
        imp, ema, da = _agent()._compute_importance_with_state(
            xt, pin["layer_index"], pin["num_layers"], attn_is_probabilities=pin["contract"] == "probs",
            received_ema=pt, irap_decay=pin["decay"], entropy_weight=pin["beta"], sink_tokens=pin["sink"])
    assert imp.shape == (pin["Sk"], pin["H"]) and imp.dtype == torch.float32 and imp.is_cuda
    assert np.abs(imp.cpu().numpy() - a["importance"]).max() <= 1e-6
    np.testing.assert_allclose(ema.cpu().numpy(), a["ema"], rtol=1e-6, atol=1e-12)
    if pin["delta_a"] is None:
        assert da is None
    else:
        assert abs(da - pin["delta_a"]) <= 1e-5 * abs(pin["delta_a"])


@pytest.mark.parametrize("B,H,Sq,Sk,kind,contract,prev_len,beta,sink", [
    (1, 8, 1024, 1024, "probs", None, 900, 0.3, 4),
    (2, 4, 500, 700, "logits", "logits", None, 0.5, 0),
    (1, 6, 333, 258, "raw", "probs", 300, 0.0, 300),   # Sk not a multiple of 4; sinks cover all
    (1, 3, 64, 2100, "probs", None, 2100, 1.0, 2),     # three key tiles, bitonic sort of 4096 slots
    (1, 2, 8, 16500, "probs", None, 16000, 0.3, 4),    # beyond the shared-memory sort: counting ranks
])
def test_irap_matches_oracle(skv, B, H, Sq, Sk, kind, contract, prev_len, beta, sink):
    x = irap_scores(Sq + Sk, B, H, Sq, Sk, kind=kind)
    prev = None
    if prev_len:
        prev = (np.random.default_rng(3).random((prev_len, H)) / Sk).astype(np.float32)
    xo = x if contract is None else DO.irap_inputs(x, contract == "probs")
    oi, oe, oda = DO.compute_irap_importance(xo, prev, 0.9, beta, sink, 1, 4)
    xt = torch.from_numpy(x).cuda()
    pt = None if prev is None else torch.from_numpy(prev).cuda()
    if contract is None:
        gi, ge, gda = skv.compute_irap_importance(xt, pt, 0.9, beta, sink, 1, 4)
    else:
        gi, ge, gda = _agent()._compute_importance_with_state(xt, 1, 4, attn_is_probabilities=contract == "probs",
                                                              received_ema=pt, entropy_weight=beta,
                                                              sink_tokens=sink)
    diff = np.abs(gi.cpu().numpy() - oi)
    # probabilities as given: compensated sums, EMA to a couple of ulp; through the contract
    # the softmax / row correction rounds differently (GPU float32 vs oracle float64), 2e-6
    rel = 2.5e-7 if contract is None else 2e-6
    np.testing.assert_allclose(ge.cpu().numpy(), oe, rtol=rel, atol=1e-12)
    # tokens whose EMA is that close to another token's of the same head may swap ranks
    # (one rank step = (1 - beta) / Sk * layer factor); all others within 1e-6
    near = _near_ties(oe, 2 * rel)
    assert diff[~near].max(initial=0.0) <= 1e-6
    step = (1.0 - beta) / Sk * (1.0 + 0.1 * 0.25)
    assert diff[near].max(initial=0.0) <= 2 * step + 1e-6
    assert (gda is None) == (oda is None)
    if oda is not None:
        assert abs(gda - oda) <= 1e-6 * abs(oda)


def _near_ties(ema: np.ndarray, rel: float) -> np.ndarray:
    """[Sk,H] bool: tokens whose EMA is within ``rel`` (relative) of a neighbour in sorted order."""
    out = np.zeros(ema.shape, bool)
    for h in range(ema.shape[1]):
        col = ema[:, h].astype(np.float64)
        order = np.argsort(col, kind="stable")
        sv = col[order]
        close = np.abs(np.diff(sv)) <= rel * np.maximum(np.abs(sv[1:]), 1e-30)
        flag = np.zeros(len(sv), bool)
        flag[1:] |= close
        flag[:-1] |= close
        out[order, h] = flag
    return out


def test_irap_ties_rank_by_token_index(skv):
    """Exactly equal EMA values (tokens nobody attends to) are ranked in token order."""
    x = np.zeros((1, 2, 16, 40), np.float32)
    x[:, :, :, 30:] = 0.1                            # tokens 0..29 receive nothing: a 30-way tie
    imp, ema, _ = skv.compute_irap_importance(torch.from_numpy(x).cuda(), entropy_weight=0.0, sink_tokens=0)
    expected = ((np.arange(40) + 1.0) / 40.0).astype(np.float32)
    for h in range(2):
        assert np.array_equal(imp.cpu().numpy()[:, h], expected)


def test_irap_validation_errors(skv):
    w = torch.rand(1, 2, 4, 4, device="cuda")
    with pytest.raises(ValueError, match="4-D"):
        skv.compute_irap_importance(w[0])
    with pytest.raises(ValueError, match="irap_decay"):
        skv.compute_irap_importance(w, irap_decay=1.0)
    with pytest.raises(ValueError, match="entropy_weight"):
        skv.compute_irap_importance(w, entropy_weight=1.5)
    with pytest.raises(ValueError, match="sink_tokens"):
        skv.compute_irap_importance(w, sink_tokens=-1)
