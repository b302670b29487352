"""CPU: the oracle restatements pinned against the reference's golden vectors."""

import hashlib
import json
import os

import numpy as np
import pytest
import torch

from cast_b200 import workloads
from oracle import par as opar
from oracle import rcsa as orc

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _sha(a) -> str:
    if isinstance(a, torch.Tensor):
        a = a.view(torch.int16) if a.dtype == torch.bfloat16 else a
        a = a.numpy()
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_manifest_hashes():
    man = json.load(open(os.path.join(GOLDEN, "MANIFEST.json")))
    for f, h in man["files"].items():
        with open(os.path.join(GOLDEN, f), "rb") as fh:
            assert hashlib.sha256(fh.read()).hexdigest() == h, f


def test_workload_generators_reproduce_golden_inputs():
    man = json.load(open(os.path.join(GOLDEN, "MANIFEST.json")))["inputs"]
    w = workloads.config1()
    assert _sha(w.meta["q_full"]) == man["config1"]["q_full"]
    assert _sha(w.k) == man["config1"]["k"] and _sha(w.v) == man["config1"]["v"]
    w3 = workloads.config3(heads=2)
    assert [_sha(t) for t in (w3.q, w3.k, w3.v)] == [man["config3_h2"][n] for n in "qkv"]
    assert _sha(workloads.config4(channels=64).full_residual) == man["par_c64"]["full_residual"]
    assert _sha(workloads.par_motion(channels=64).full_residual) == man["par_motion_c64"]["full_residual"]


def test_taba_select_matches_reference_select():
    """Oracle TABA selection == MatrixTrajectoryAdaptiveBudgetAttentionCompiler.select."""
    g = np.load(os.path.join(GOLDEN, "cfg1_select.npz"))
    w = workloads.config1()
    sel, cnt, _ = orc.taba_select(w.meta["q_full"].numpy(), w.k.numpy(), (8, 8), (1, 8, 8),
                                  g["taba_row_degrees"])
    assert np.array_equal(sel, g["taba_selected"])
    assert np.array_equal(cnt, g["taba_counts"])


def test_budget_rule_matches_reference_primitives_config1():
    g = np.load(os.path.join(GOLDEN, "cfg1_select.npz"))
    w = workloads.config1()
    sel, cnt, _, _, scores = orc.rcsa_select(w.q.numpy(), w.k.numpy(), 64, 4)
    assert np.array_equal(sel, g["budget_selected"]) and np.array_equal(cnt, g["budget_counts"])
    assert np.abs(scores - g["budget_scores_f32"]).max() < 1e-5
    # the kernels take bf16 inputs: selection is unchanged by bf16 rounding here
    sel16, _, _, _, _ = orc.rcsa_select(w.q.bfloat16().float().numpy(),
                                        w.k.bfloat16().float().numpy(), 64, 4)
    assert np.array_equal(sel16, g["budget_selected"])


def test_budget_rule_matches_reference_primitives_config2_two_heads():
    g = np.load(os.path.join(GOLDEN, "cfg2_select_h2.npz"))
    w = workloads.config2(heads=24)
    q = w.q[:, :2].float().numpy()
    k = w.k[:, :2].float().numpy()
    sel, cnt, _, _, scores = orc.rcsa_select(q, k, 880, 8)
    assert np.array_equal(sel, g["selected"]) and np.array_equal(cnt, g["counts"])
    assert np.abs(scores - g["scores_f32"]).max() < 1e-5


def test_budget_rule_matches_reference_primitives_config3():
    """Anchor-only queries over a 128-frame history, budget 16."""
    g = np.load(os.path.join(GOLDEN, "cfg3_select_h2.npz"))
    w = workloads.config3(heads=2)
    sel, cnt, _, _, scores = orc.rcsa_select(w.q.float().numpy(), w.k.float().numpy(), 880, w.budget)
    assert np.array_equal(sel, g["selected"]) and np.array_equal(cnt, g["counts"])
    assert np.abs(scores - g["scores_f32"]).max() < 1e-5


def test_quantiser_and_attention_golden_config1():
    g = np.load(os.path.join(GOLDEN, "cfg1_quant_attn.npz"))
    gs = np.load(os.path.join(GOLDEN, "cfg1_select.npz"))
    w = workloads.config1()
    qc, qs = orc.quantize_blocks(w.q.numpy(), 64)
    kc, ks = orc.quantize_blocks(w.k.numpy(), 64)
    vc, vs = orc.quantize_blocks(w.v.numpy(), 64)
    assert np.array_equal(qs, g["q_scales"]) and np.array_equal(ks, g["k_scales"])
    assert np.array_equal(vs, g["v_scales"])
    assert _sha(qc) == str(g["q_codes_sha"]) and _sha(kc) == str(g["k_codes_sha"])
    assert _sha(vc) == str(g["v_codes_sha"])
    q16, k16, v16 = (t.bfloat16().float().numpy() for t in (w.q, w.k, w.v))
    o = orc.block_sparse_attention(q16, k16, v16, gs["budget_selected"], gs["budget_counts"], 64, 64)
    assert np.abs(o - g["attn_bf16"]).max() < 1e-6


def test_quantiser_definition_edge_cases():
    x = np.zeros((1, 1, 4, 32), dtype=np.float32)
    codes, s = orc.quantize_blocks(x, 4)
    assert s[0, 0, 0] == 1.0 and not codes.any()  # amax == 0 -> scale 1
    x[0, 0, 0, :3] = [1.0, -1.0, 0.5]
    codes, s = orc.quantize_blocks(x, 4)
    assert codes[0, 0, 0, 0] == 127 and codes[0, 0, 0, 1] == -127
    assert codes[0, 0, 0, 2] == 64  # 0.5/(1/127) = 63.5 -> half to even = 64


def test_par_restatement_matches_reference_golden():
    for name, wl in (("par_c64", workloads.config4(channels=64)),
                     ("par_motion_c64", workloads.par_motion(channels=64))):
        g = np.load(os.path.join(GOLDEN, f"{name}.npz"))
        out, inter = opar.correct(wl.full_residual.float().numpy(), wl.active_residual.float().numpy(),
                                  wl.active_frames, wl.memory_length, 22, 40, return_intermediates=True)
        got = torch.from_numpy(out[0, list(g["target_frames"])]).to(torch.bfloat16).float()
        ref = torch.from_numpy(g["targets_bf16_bits"]).view(torch.bfloat16).float()
        d = (got - ref).abs()
        assert float(d.max()) < 1e-3, name
        st = inter["stats"][(0, 3)]
        np.testing.assert_allclose(st["base_confidence"], g["stats_base_confidence"], atol=1e-4)
        np.testing.assert_allclose(st["ramp_confidence"], g["stats_ramp_confidence"], atol=1e-4)
        np.testing.assert_allclose(st["displacement"], g["stats_displacement"], atol=1e-3)


def test_par_known_answer_identities():
    """g = 0 gives the linear spectral mix and g = 1 the PASM shift
    (proposed/matrix_world_spectral_residual.py:3405-3422); OLA covers every
    pixel (:2046-2047)."""
    rng = np.random.default_rng(0)
    left = rng.normal(size=(18, 4, 11, 6)) + 1j * rng.normal(size=(18, 4, 11, 6))
    right = rng.normal(size=(18, 4, 11, 6)) + 1j * rng.normal(size=(18, 4, 11, 6))
    theta = rng.uniform(-np.pi, np.pi, size=(18, 11, 6))
    a = 0.25
    m0 = opar.mix(left, right, theta, np.zeros_like(theta), a)
    np.testing.assert_allclose(m0, (1 - a) * left + a * right, atol=1e-12)
    m1 = opar.mix(left, right, theta, np.ones_like(theta), a)
    exp = (1 - a) * left * np.exp(1j * a * theta)[:, None] + a * right * np.exp(-1j * (1 - a) * theta)[:, None]
    np.testing.assert_allclose(m1, exp, atol=1e-12)
    assert opar.ola_normalization(22, 40, opar.overlap_window()).min() > 1e-8


def test_fast_quantiser_matches_ieee_division_exhaustively(tmp_path):
    """The kernel's division-free quantiser (Markstein-corrected quotient)
    gives the defined code for every bf16 amax and bf16 |x| <= amax."""
    import shutil
    import subprocess

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    src = os.path.join(os.path.dirname(__file__), "quant_fastpath_exhaustive.c")
    exe = str(tmp_path / "quant_fastpath_exhaustive")
    subprocess.run([cc, "-O2", "-ffp-contract=off", "-o", exe, src, "-lm"], check=True)
    res = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "mismatches 0" in res.stdout and "out of range 0" in res.stdout


@pytest.mark.parametrize("name", ["cfg2", "cfg3"])
def test_budget_rule_matches_reference_primitives_all_heads(name):
    """All 24 heads of config 2, and config 3 generated with 24 heads: the
    oracle's selection equals the one built from the reference's own pooling
    primitives (``cfg*_select_h24.npz``)."""
    w = workloads.config2() if name == "cfg2" else workloads.config3(heads=24)
    sel, cnt, _, _, _ = orc.rcsa_select(w.q.float().numpy(), w.k.float().numpy(), 880, w.budget)
    g = np.load(os.path.join(GOLDEN, f"{name}_select_h24.npz"))
    np.testing.assert_array_equal(sel, g["selected"])
    np.testing.assert_array_equal(cnt, g["counts"])


def _compact_golden(name):
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLDEN, "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    frames, mem, active, shape, heads, _, _ = mg.COMPACT_SELECT_CASES[name]
    q, k, v = mg.compact_select_case(name)
    g = np.load(os.path.join(GOLDEN, f"compact_select_{name}.npz"))
    tt, th, tw = shape
    nh, nw = -(-22 // th), -(-40 // tw)
    cells = g["block_indices"].shape[0] // (nh * nw)
    return q, k, v, g, (cells, nh, nw)


@pytest.mark.parametrize("name", ["uniform", "curved", "tt2"])
def test_compact_select_matches_reference(name):
    """The compact-path ranking restated in the oracle equals the selection
    the reference's ``_compact_cwca_attention`` handed to its attention launch."""
    q, k, _, g, grid = _compact_golden(name)
    bi = g["block_indices"]
    qp = orc.compact_pack(q.float().numpy(), bi)
    kp = orc.compact_pack(k.float().numpy(), bi)
    valid = g["valid"].reshape(-1)
    degrees = g["counts"][0, 0]
    sel, cnt, _ = orc.compact_select(qp, kp, valid, bi.shape[1], grid, degrees)
    np.testing.assert_array_equal(cnt, g["counts"])
    assert_same_rows(sel, g["selected"], cnt)


def assert_same_rows(sel, ref, cnt):
    """Every row selects the same blocks.  The stencil's 1e6 bonus, added in
    float32, rounds the local blocks' ranks onto a 1/16 grid where they tie;
    ``torch.topk`` (frame_weave.py:5831) leaves the order of tied entries to
    its implementation, the kernels and the oracle order them by index.  The
    local blocks always sit inside a row's count, so the tie order never
    changes which blocks a row attends to."""
    k = sel.shape[-1]
    in_count = np.arange(k)[None, None, None] < cnt[..., None]
    ours = np.sort(np.where(in_count, sel, -1), axis=-1)
    theirs = np.sort(np.where(in_count, ref, -1), axis=-1)
    np.testing.assert_array_equal(ours, theirs)


def _make_golden():
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLDEN, "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    return mg


@pytest.mark.parametrize("name", ["current_only", "memory_boundary", "no_controls", "memory_split"])
def test_lift_matches_reference(name):
    """The control-barycentric lift restated in the oracle (camera and action
    state, clamped cosines, softmax with the temporal prior, the two-anchor
    contraction) reproduces the reference's target rows."""
    from oracle import barycentric as obary
    mg = _make_golden()
    frames, mem, active, boundary, _, _, lambdas, _ = mg.LIFT_CASES[name]
    act, af, plucker, mouse, keyboard, mm, km = mg.lift_case(name)
    npy = lambda x: None if x is None else x[0].float().numpy()  # noqa: E731
    full, w, targets = obary.lift(npy(act), list(active), frames, mem, boundary, npy(plucker), npy(mouse),
                                  npy(keyboard), npy(mm), npy(km), lambdas)
    g = np.load(os.path.join(GOLDEN, f"lift_{name}.npz"))
    assert [t[0] for t in targets] == list(g["targets"])
    assert int(g["n_targets"]) == len(targets)
    np.testing.assert_allclose(full[g["targets"]], g["target_rows"], rtol=0, atol=2e-6)
    np.testing.assert_allclose(w.sum(-1), 1.0, atol=1e-6)
