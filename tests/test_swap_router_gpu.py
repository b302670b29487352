"""FC-PASM swap router on the B200: the CUDA path (``cast_swap_route``)
against the reference's own ``refine`` outputs (golden fixtures) and against
the CPU oracle at a layer-sized case."""

import numpy as np
import pytest
import torch

from cast_b200 import _lib, workloads
from cast_b200 import swap_router as sr
from oracle import swap_router as osr

from test_swap_router import CASES, _fixture, oracle_refine

pytestmark = pytest.mark.gpu


def _to(w, dev):
    for name in ("score", "pooled_value", "selected", "counts", "local"):
        setattr(w, name, getattr(w, name).to(dev))
    if w.transport is not None:
        for e in w.transport["pairs"].values():
            e["theta"], e["affinity"] = e["theta"].to(dev), e["affinity"].to(dev)
    return w


def _refine(router, w):
    return router.refine(score=w.score, pooled_value=w.pooled_value, selected=w.selected.clone(),
                         counts=w.counts, local=w.local, memory_blocks=w.memory_blocks,
                         spatial_shape=w.spatial_shape, exact_current_frames=w.exact_frames,
                         temporal_group_size=w.temporal_group_size, current_boundary=w.current_boundary,
                         transport=w.transport, layer_index=22)


@pytest.mark.parametrize("name", sorted(CASES))
def test_refine_matches_reference(name):
    case_kw, cfg_kw = CASES[name]
    w = _to(workloads.swap_case(**case_kw), "cuda")
    fx = _fixture(name)
    router = sr.FCPASMLocalCoordinateSwapRouter(sr.FCPASMSwapRoutingConfig(**cfg_kw))
    sel, rec = _refine(router, w)
    assert rec["status"] == str(fx["status"])
    np.testing.assert_array_equal(sel.cpu().numpy(), fx["selected_after"])
    assert rec["swap_count"] == int(fx["swap_count"])
    # objectives: fp32 terms summed in another order (fp64 on the device)
    assert float(rec["objective_before"]) == pytest.approx(float(fx["objective_before"]), rel=1e-4)
    assert float(rec["objective_after"]) == pytest.approx(float(fx["objective_after"]), rel=1e-4)
    assert _lib.load().cast_device_error(None) == 0


def _layer_case(seed=21):
    # a 24-head layer: 32 memory blocks, 4 current cells of 2x4 blocks, D=128
    return workloads.swap_case(heads=24, memory_blocks=32, cells=4, spatial_shape=(2, 4), dim=128,
                               width=16, exact_frames=(0, 3), transport=True, seed=seed)


@pytest.mark.parametrize("rounds,eps", [(1, 0.0), (2, 1e-6)])
def test_layer_case_matches_oracle(rounds, eps):
    w = _layer_case()
    ops = {}

    def op(pair, x):
        key = (pair, round(float(x), 12))
        if key not in ops:
            ops[key] = sr.transport_operator(w.transport, pair, spatial_shape=w.spatial_shape,
                                             exponent=x, device="cpu")[0].numpy()
        return ops[key]

    cfg = dict(num_swap_rounds=rounds, swap_eps=eps)
    sel_o, st = osr.refine(score=w.score.numpy(), pooled_value=w.pooled_value.numpy(),
                           selected=w.selected.numpy(), counts=w.counts.numpy(), local=w.local.numpy(),
                           memory_blocks=w.memory_blocks, spatial=8, exact_frames=w.exact_frames,
                           group=1, boundary=4, config=osr.SwapConfig(**cfg), operator=op)
    wd = _to(_layer_case(), "cuda")
    router = sr.FCPASMLocalCoordinateSwapRouter(sr.FCPASMSwapRoutingConfig(**cfg))
    sel, rec = _refine(router, wd)
    assert st["swap_count"] >= 1
    assert rec["swap_count"] == st["swap_count"]
    np.testing.assert_array_equal(sel.cpu().numpy(), sel_o)
    assert float(rec["objective_before"]) == pytest.approx(st["objective_before"], rel=1e-4)
    assert float(rec["objective_after"]) == pytest.approx(st["objective_after"], rel=1e-4)


def test_oracle_fixture_helper_on_device_inputs():
    """The oracle path the GPU tests lean on agrees with the fixture too."""
    case_kw, cfg_kw = CASES["fc_two_rounds"]
    w = workloads.swap_case(**case_kw)
    sel, st = oracle_refine(w, cfg_kw, _fixture("fc_two_rounds"))
    np.testing.assert_array_equal(sel, _fixture("fc_two_rounds")["selected_after"])


def test_c_abi_rejects_bad_arguments():
    lib = _lib.load()
    dev = "cuda"
    w = _to(workloads.swap_case(), dev)
    stats = torch.empty(14, dtype=torch.float64, device=dev)
    coef = torch.zeros(32, device=dev)
    hess = torch.zeros(32, 32, device=dev)
    sel = w.selected.clone()
    B, H, Q, K = w.score.shape
    nbytes = lib.cast_swap_route_workspace_bytes(B, H, Q, K, 64, 10, 6, 2, 0, 16)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)

    def call(**over):
        a = dict(G=16, rounds=1, M=6, ws=ws.numel(), mult=2)
        a.update(over)
        return lib.cast_swap_route(w.score.data_ptr(), w.pooled_value.data_ptr(), sel.data_ptr(),
                                   w.counts.data_ptr(), w.local.to(torch.uint8).data_ptr(), None,
                                   None, coef.data_ptr(), hess.data_ptr(), B, H, Q, K, 64, 10, a["M"], a["mult"],
                                   a["rounds"], 0.0, a["G"], 0, 0, 0, stats.data_ptr(), ws.data_ptr(),
                                   a["ws"], None)

    assert call(G=3) != 0          # odd sketch groups
    assert call(G=24) != 0         # D not divisible
    assert call(rounds=3) != 0
    assert call(M=Q) != 0          # no current rows
    assert call(mult=0) != 0
    assert call(ws=16) != 0        # workspace too small
    torch.cuda.synchronize()
    assert torch.equal(sel, w.selected)


def test_swap_route_graph_rate():
    """One layer-sized call (proxy + one round + close) replayed from a CUDA
    graph: reports the per-call device time."""
    w = _to(_layer_case(), "cuda")
    lib = _lib.load()
    B, H, Q, K = w.score.shape
    D, S, M = w.pooled_value.shape[-1], w.selected.shape[-1], w.memory_blocks
    coef, hess, _ = sr.quadratic_terms(temporal_cells=4, spatial=8, exact_frames=(0, 3),
                                       temporal_group_size=1, current_boundary=4, transport=w.transport,
                                       lambda_anchor=1.0, lambda_reconstruction=1.0, device="cuda")
    nbytes = lib.cast_swap_route_workspace_bytes(B, H, Q, K, D, S, M, 2, 0, 16)
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    stats = torch.empty(14, dtype=torch.float64, device="cuda")
    local = w.local.to(torch.uint8)
    sel = w.selected.clone()
    s = torch.cuda.Stream()

    def launch():
        _lib.call("cast_swap_route", w.score.data_ptr(), w.pooled_value.data_ptr(), sel.data_ptr(),
                  w.counts.data_ptr(), local.data_ptr(), None, None, coef.data_ptr(), hess.data_ptr(), B, H, Q,
                  K, D, S, M, 2, 1, 0.1, 16, 1, 0, 1, stats.data_ptr(), ws.data_ptr(), nbytes,
                  s.cuda_stream)

    with torch.cuda.stream(s):
        launch()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for _ in range(20):
            launch()
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / 20
    print(f"swap route, 24 heads x 32 current rows, 64 keys, D=128: {us:.1f} us per call")
    assert us < 1000.0


def _oracle_op(w):
    ops = {}

    def op(pair, x):
        key = (pair, round(float(x), 12))
        if key not in ops:
            ops[key] = sr.transport_operator(w.transport, pair, spatial_shape=w.spatial_shape,
                                             exponent=x, device="cpu")[0].numpy()
        return ops[key]
    return op


def _short_rows_case(historical_only: bool, seed: int = 5):
    """A layer case whose rows are all shorter than the selection width, so the
    reference's candidate width min(cand_blocks, 2 * max swappable count) is
    below the device's 2 * S slots.  Historical-only: each current row's
    non-local keys are random memory blocks, so selected keys rank past that
    width in the candidate order (their proxies must then count as zero)."""
    w = _layer_case(seed=seed)
    g = torch.Generator().manual_seed(seed)
    B, H, Q, K = w.score.shape
    S, M = w.selected.shape[-1], w.memory_blocks
    sel = w.selected.clone()
    counts = w.counts.clone()
    if historical_only:
        for h in range(H):
            for q in range(M, Q):
                n_local = int(w.local[q].sum())
                pick = torch.randperm(M, generator=g)[: S - n_local]
                sel[0, h, q, n_local:] = pick
        counts[:] = S - 3 - torch.randint(0, 3, counts.shape, generator=g)
    else:
        counts[:] = S - 4 - torch.randint(0, 3, counts.shape, generator=g)
    slot = torch.arange(S)[None, None, None]
    pad = torch.gather(sel, -1, (counts - 1)[..., None])
    w.selected = torch.where(slot < counts[..., None], sel, pad)
    w.counts = counts
    return w


@pytest.mark.parametrize("historical_only", [False, True])
def test_short_rows_match_oracle(historical_only):
    """Rows shorter than the selection width: the removed key's proxy is looked
    up only within the reference's candidate width (fc_pasm_swap_routing.py:
    820-826); beyond it the proxy is zero, on the device as in the oracle."""
    w = _short_rows_case(historical_only)
    cfg = dict(num_swap_rounds=2, swap_eps=0.0, historical_only=historical_only)
    sel_o, st = osr.refine(score=w.score.numpy(), pooled_value=w.pooled_value.numpy(),
                           selected=w.selected.numpy(), counts=w.counts.numpy(), local=w.local.numpy(),
                           memory_blocks=w.memory_blocks, spatial=8, exact_frames=w.exact_frames,
                           group=1, boundary=4, config=osr.SwapConfig(**cfg), operator=_oracle_op(w))
    wd = _to(_short_rows_case(historical_only), "cuda")
    router = sr.FCPASMLocalCoordinateSwapRouter(sr.FCPASMSwapRoutingConfig(**cfg))
    sel, rec = _refine(router, wd)
    assert rec["status"] == "refined"
    assert rec["swap_count"] == st["swap_count"]
    np.testing.assert_array_equal(sel.cpu().numpy(), sel_o)
    assert float(rec["objective_before"]) == pytest.approx(st["objective_before"], rel=1e-4)
    assert float(rec["objective_after"]) == pytest.approx(st["objective_after"], rel=1e-4)
    assert rec["candidate_max"] == st["candidate_max"] < 2 * w.selected.shape[-1]


@pytest.mark.parametrize("frames,group,cells", [((0, 3), 1, 4), ((0, 3, 4, 7), 1, 8), ((0, 2, 5), 2, 3)])
def test_device_objective_matches_host_restatement(cuda, frames, group, cells):
    """cast_swap_objective's coefficient vector and Hessian against the torch
    restatement of the reference's per-call construction (transport
    operators from the sketch, then the quadratic terms), with the sketch
    published for some pairs and missing (identity operator) for others."""
    w = workloads.swap_case(transport=True, exact_frames=frames, cells=cells, temporal_group_size=group,
                            width=12, seed=8)
    pairs = w.transport["pairs"]
    if len(pairs) > 1:  # one pair without a sketch: identity operators
        pairs.pop(sorted(pairs)[-1])
    coef_ref, hess_ref, _ = sr.quadratic_terms(
        temporal_cells=cells, spatial=8, exact_frames=frames, temporal_group_size=group,
        current_boundary=4, transport=w.transport, lambda_anchor=1.0, lambda_reconstruction=0.7,
        device="cpu")
    for e in pairs.values():
        for name in ("theta", "affinity", "mean_affinity"):
            e[name] = e[name].cuda()
    router = sr.FCPASMLocalCoordinateSwapRouter(sr.FCPASMSwapRoutingConfig(lambda_reconstruction=0.7))
    stats = torch.zeros(14, dtype=torch.float64, device="cuda")
    same_seg = [(a, b) for a, b in zip(frames, frames[1:]) if (a < 4) == (b < 4)]
    obj = router._objective(cells=cells, spatial=8, spatial_shape=(2, 4), frames=frames, same_seg=same_seg,
                            pairs=pairs, transport=w.transport, group=group, boundary=4, stats=stats,
                            device=torch.device("cuda"), stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    np.testing.assert_allclose(obj["coef"].cpu().numpy(), coef_ref.numpy(), rtol=1e-6)
    scale = float(hess_ref.abs().max())
    assert float((obj["hess"].cpu() - hess_ref).abs().max()) < 1e-5 * scale
    assert int(stats[5]) == 0 and obj["sketched"] == bool(pairs)


def test_device_gates(cuda):
    """The transport gates on the device: a sketch below the matching gate,
    and a pair gate that no pair passes, give the reference's fallbacks and
    leave the selection as it is."""
    w = _to(workloads.swap_case(transport=True), "cuda")
    for e in w.transport["pairs"].values():
        e["mean_affinity"] = torch.tensor(0.3, device="cuda")
    for cfg, reason in ((dict(require_fc_transport=True, min_transport_affinity=0.5),
                         "weak_previous_layer_fc_transport"),
                        (dict(min_pair_transport_affinity=0.5), "no_strong_transport_pair_cells")):
        router = sr.FCPASMLocalCoordinateSwapRouter(sr.FCPASMSwapRoutingConfig(num_swap_rounds=2, **cfg))
        sel, rec = _refine(router, w)
        assert rec["status"] == "independent_topk_fallback" and rec["fallback_reason"] == reason
        assert rec["matching_transport_affinity"] == pytest.approx(0.3)
        assert torch.equal(sel, w.selected)
    # the same sketch above both gates refines
    for e in w.transport["pairs"].values():
        e["mean_affinity"] = torch.tensor(0.8, device="cuda")
    router = sr.FCPASMLocalCoordinateSwapRouter(sr.FCPASMSwapRoutingConfig(
        num_swap_rounds=2, require_fc_transport=True, min_transport_affinity=0.5,
        min_pair_transport_affinity=0.5))
    _, rec = _refine(router, w)
    assert rec["status"] == "refined" and rec["pair_gate_cells"] >= 1
