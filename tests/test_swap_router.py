"""FC-PASM swap router: the CPU oracle against the reference's own ``refine``
outputs, and the host-side pieces of the B200 router (transport operators,
quadratic terms, configuration checks, fallback records)."""

import hashlib
import importlib.util
import json
import os

import numpy as np
import pytest
import torch

from cast_b200 import swap_router as sr
from cast_b200 import workloads
from oracle import swap_router as osr

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")


def _cases():
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLDEN, "make_golden.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.SWAP_CASES


CASES = _cases()


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _fixture(name):
    return np.load(os.path.join(GOLDEN, f"swap_{name}.npz"))


def _operator_table(fx):
    table = {(int(k[0]), int(k[1]), round(float(k[2]), 12)): m for k, m in zip(fx["op_keys"], fx["ops"])}
    return lambda pair, x: table[(pair[0], pair[1], round(float(x), 12))]


def _oracle_config(cfg_kw):
    fields = osr.SwapConfig.__dataclass_fields__
    return osr.SwapConfig(**{k: v for k, v in cfg_kw.items() if k in fields})


def oracle_refine(w, cfg_kw, fx):
    op = _operator_table(fx) if w.transport is not None else None
    sp = w.spatial_shape[0] * w.spatial_shape[1]
    cells = (w.score.shape[2] - w.memory_blocks) // sp
    gate = None
    if cfg_kw.get("min_pair_transport_affinity", 0.0) > 0.0:
        pairs = w.transport["pairs"]
        gate = osr.pair_row_gate(
            exact_frames=w.exact_frames, boundary=w.current_boundary, group=w.temporal_group_size,
            cells=cells, spatial=sp, threshold=cfg_kw["min_pair_transport_affinity"],
            affinity_of=lambda p: float(pairs[p]["mean_affinity"]) if p in pairs else 0.0)
    return osr.refine(score=w.score.numpy(), pooled_value=w.pooled_value.numpy(),
                      selected=w.selected.numpy(), counts=w.counts.numpy(), local=w.local.numpy(),
                      memory_blocks=w.memory_blocks, spatial=sp, exact_frames=w.exact_frames,
                      group=w.temporal_group_size, boundary=w.current_boundary,
                      config=_oracle_config(cfg_kw), operator=op, row_gate=gate)


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_matches_reference_refine(name):
    case_kw, cfg_kw = CASES[name]
    w = workloads.swap_case(**case_kw)
    with open(os.path.join(GOLDEN, "MANIFEST.json")) as fh:
        inputs = json.load(fh)["inputs"]
    for tag, t in (("score", w.score), ("value", w.pooled_value), ("selected", w.selected),
                   ("counts", w.counts)):
        assert _sha(t.numpy()) == inputs[f"swap_{name}_{tag}"], f"{tag} input drifted"
    fx = _fixture(name)
    sel, st = oracle_refine(w, cfg_kw, fx)
    np.testing.assert_array_equal(sel, fx["selected_after"])
    assert st["swap_count"] == int(fx["swap_count"])
    assert st["objective_before"] == pytest.approx(float(fx["objective_before"]), rel=1e-5)
    assert st["objective_after"] == pytest.approx(float(fx["objective_after"]), rel=1e-5)


@pytest.mark.parametrize("name", ["fc_production", "pair_gate"])
def test_transport_operator_matches_reference(name):
    case_kw, _ = CASES[name]
    w = workloads.swap_case(**case_kw)
    fx = _fixture(name)
    assert len(fx["ops"]) > 0
    for (left, right, x), ref in zip(fx["op_keys"], fx["ops"]):
        op, used = sr.transport_operator(w.transport, (int(left), int(right)),
                                         spatial_shape=w.spatial_shape, exponent=float(x), device="cpu")
        assert used
        np.testing.assert_allclose(op.numpy(), ref, rtol=1e-5, atol=1e-6)


def test_transport_operator_identity_without_sketch():
    op, used = sr.transport_operator(None, (0, 3), spatial_shape=(2, 4), exponent=0.5, device="cpu")
    assert not used and torch.equal(op, torch.eye(8))
    w = workloads.swap_case(transport=True)
    op, used = sr.transport_operator(w.transport, (0, 2), spatial_shape=(2, 4), exponent=0.5, device="cpu")
    assert not used and torch.equal(op, torch.eye(8))
    # exponent zero is the identity up to the round trip's rounding
    op, used = sr.transport_operator(w.transport, (0, 3), spatial_shape=(2, 4), exponent=0.0, device="cpu")
    assert used
    np.testing.assert_allclose(op.numpy(), np.eye(8), atol=1e-6)


@pytest.mark.parametrize("name", sorted(CASES))
def test_quadratic_terms_match_oracle(name):
    case_kw, cfg_kw = CASES[name]
    w = workloads.swap_case(**case_kw)
    fx = _fixture(name)
    sp = w.spatial_shape[0] * w.spatial_shape[1]
    cells = (w.score.shape[2] - w.memory_blocks) // sp
    coef, hess, used = sr.quadratic_terms(
        temporal_cells=cells, spatial=sp, exact_frames=w.exact_frames,
        temporal_group_size=w.temporal_group_size, current_boundary=w.current_boundary,
        transport=w.transport, lambda_anchor=1.0, lambda_reconstruction=1.0, device="cpu")
    c, H = osr.quadratic_terms(cells=cells, spatial=sp, exact_frames=w.exact_frames,
                               group=w.temporal_group_size, boundary=w.current_boundary, lam_a=1.0,
                               lam_r=1.0, operator=_operator_table(fx) if w.transport else None)
    assert used == (w.transport is not None)
    np.testing.assert_allclose(coef.numpy(), c, rtol=1e-6)
    np.testing.assert_allclose(hess.numpy(), H, rtol=1e-5, atol=1e-6)


def test_config_checks_mirror_reference_messages():
    with pytest.raises(ValueError, match="candidate multiplier must be positive"):
        sr.FCPASMSwapRoutingConfig(candidate_multiplier=0)
    with pytest.raises(ValueError, match="zero to two swap rounds"):
        sr.FCPASMSwapRoutingConfig(num_swap_rounds=3)
    with pytest.raises(ValueError, match="positive even number"):
        sr.FCPASMSwapRoutingConfig(sketch_groups=3)
    with pytest.raises(ValueError, match="already fixes the KV bank"):
        sr.FCPASMSwapRoutingConfig(historical_only=True, same_bank_only=True)
    with pytest.raises(ValueError, match="finite and non-negative"):
        sr.FCPASMSwapRoutingConfig(swap_eps=float("nan"))


def _refine(router, w, **over):
    kw = dict(score=w.score, pooled_value=w.pooled_value, selected=w.selected.clone(), counts=w.counts,
              local=w.local, memory_blocks=w.memory_blocks, spatial_shape=w.spatial_shape,
              exact_current_frames=w.exact_frames, temporal_group_size=w.temporal_group_size,
              current_boundary=w.current_boundary, transport=w.transport, layer_index=22)
    kw.update(over)
    return router.refine(**kw)


@pytest.mark.parametrize("cfg,over,reason", [
    (dict(active_layers=(26,)), {}, "layer_not_enabled"),
    (dict(num_swap_rounds=0), {}, "zero_swap_rounds"),
    ({}, dict(exact_current_frames=(1,)), "fewer_than_two_exact_anchors"),
    ({}, dict(exact_current_frames=(0, 1, 2)), "no_skipped_frames"),
    ({}, dict(memory_blocks=7), "no_rectangular_current_rows"),
    (dict(require_fc_transport=True), dict(transport=None), "missing_previous_layer_fc_transport"),
])
def test_fallback_records(cfg, over, reason):
    """The host-only gates run before any device work, as in the reference
    (proposed/fc_pasm_swap_routing.py:636-760); the two gates on the
    sketches' mean affinities run on the device (tests/test_swap_router_gpu.py)."""
    w = workloads.swap_case(transport=True)
    router = sr.FCPASMLocalCoordinateSwapRouter(sr.FCPASMSwapRoutingConfig(**cfg))
    sel, rec = _refine(router, w, **over)
    assert rec["status"] == "independent_topk_fallback"
    assert rec["fallback_reason"] == reason
    assert torch.equal(sel, w.selected)
    assert router.summary()["records"][0]["fallback_reason"] == reason


def test_unsorted_anchor_frames_rejected():
    w = workloads.swap_case()
    router = sr.FCPASMLocalCoordinateSwapRouter(sr.FCPASMSwapRoutingConfig())
    with pytest.raises(ValueError, match="unique and chronological"):
        _refine(router, w, exact_current_frames=(3, 0))


def test_attach_router_keeps_original_for_host_tensors():
    """``attach_router`` replaces a weave's router ``refine`` in place; host
    tensors still reach the reference's own method, and attaching twice is a
    no-op."""
    from cast_b200 import components

    calls = []

    class FakeRouter:
        config = sr.FCPASMSwapRoutingConfig(num_swap_rounds=2)
        _records = []

        def refine(self, **kw):
            calls.append(kw["layer_index"])
            return kw["selected"], {"status": "reference"}

    class Weave:
        fc_pasm_swap_router = FakeRouter()

    weave = Weave()
    components.attach_router(weave)
    first = weave.fc_pasm_swap_router.refine
    components.attach_router(weave)
    assert weave.fc_pasm_swap_router.refine is first
    w = workloads.swap_case()
    _, rec = _refine(weave.fc_pasm_swap_router, w)
    assert rec["status"] == "reference" and calls == [22]
