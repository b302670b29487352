"""FC routing transport on the B200: PAR at layer 21 publishes the endpoint
sketch from its kernels' statistics, and the swap router at layer 22 reads
it -- against the reference's own layer-21 ``correct`` + layer-22 ``refine``
chain on the same inputs (``tests/golden/transport_*.npz``, written by
``make_golden.py --only transport``)."""

import os

import numpy as np
import pytest
import torch

from cast_b200 import par as cpar
from cast_b200 import swap_router as sr
from cast_b200 import workloads

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _golden_module():
    import importlib.util

    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLDEN, "make_golden.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


MG = _golden_module()
CASES = {name: (wl, kw) for name, wl, kw in MG.transport_cases()}


def _publish(name):
    wl, _ = CASES[name]
    c = cpar.FCPASMCorrector()
    c._fc_routing_publish_layers = frozenset({21})
    c.begin_model_call(chunk_index=1, step_index=0)
    full = wl.full_residual.clone().cuda()
    c.correct(layer_index=21, full_input=None, full_residual=full, active_residual=wl.active_residual.cuda(),
              active_frames=torch.tensor(wl.active_frames), memory_length=wl.memory_length,
              spatial_height=22, spatial_width=40, active_frame_values=tuple(wl.active_frames))
    torch.cuda.synchronize()
    return c, full, wl


@pytest.mark.parametrize("name", sorted(CASES))
def test_published_sketch_matches_reference(cuda, name):
    g = np.load(os.path.join(GOLDEN, f"transport_{name}.npz"))
    c, full, wl = _publish(name)
    assert c.fc_pasm_routing_transport(layer_index=23) is None   # only layer 21 publishes
    tr = c.fc_pasm_routing_transport(layer_index=22)
    assert tr is not None and tr["source_layer"] == 21 and tr["transport_shape"] == (11, 10)
    assert sorted(tr["pairs"]) == [tuple(int(v) for v in p) for p in g["pairs"]]
    assert list(tr["exact_frames"]) == list(g["exact_frames"])
    for (left, right), e in tr["pairs"].items():
        aff_ref = g[f"affinity_{left}_{right}"]
        aff = e["affinity"].cpu().numpy()
        assert np.abs(aff - aff_ref).max() < 2e-3
        # the phase the router applies is x * g * theta with |x| <= 1: compare
        # g * theta with the angle wrapped (ill-conditioned bins have g ~ 0)
        d = np.angle(np.exp(1j * (e["theta"].cpu().numpy() - g[f"theta_{left}_{right}"])))
        assert np.abs(d * aff_ref).max() < 2e-3
        assert float(e["mean_affinity"]) == pytest.approx(float(g[f"mean_affinity_{left}_{right}"]),
                                                          abs=2e-4)
    assert float(c._fc_previous_mean_affinity) == pytest.approx(float(g["previous_mean_affinity"]), abs=2e-4)
    got = full[0, wl.memory_length:].float().flatten()[::11].cpu().numpy()
    assert np.abs(got - g["current_sample"]).max() < 2e-3


@pytest.mark.parametrize("name", sorted(CASES))
@pytest.mark.parametrize("tag", sorted(MG.TRANSPORT_ROUTER))
def test_router_on_published_sketch_matches_reference(cuda, name, tag):
    """Layer 22's router on the sketch layer 21 published: the reference's
    status, swap count, selection and objectives."""
    g = np.load(os.path.join(GOLDEN, f"transport_{name}.npz"))
    c, _, _ = _publish(name)
    _, case_kw = CASES[name]
    w = workloads.swap_case(**case_kw)
    transport = dict(c.fc_pasm_routing_transport(layer_index=22))
    transport["attention_spatial_h"], transport["attention_spatial_w"] = w.spatial_shape
    router = sr.FCPASMLocalCoordinateSwapRouter(sr.FCPASMSwapRoutingConfig(**MG.TRANSPORT_ROUTER[tag]))
    sel, rec = router.refine(
        score=w.score.cuda(), pooled_value=w.pooled_value.cuda(), selected=w.selected.clone().cuda(),
        counts=w.counts.cuda(), local=w.local.cuda(), memory_blocks=w.memory_blocks,
        spatial_shape=w.spatial_shape, exact_current_frames=w.exact_frames,
        temporal_group_size=w.temporal_group_size, current_boundary=w.current_boundary,
        transport=transport, layer_index=22)
    assert rec["status"] == str(g[f"{tag}_status"]) == "refined"
    assert rec["swap_count"] == int(g[f"{tag}_swap_count"])
    np.testing.assert_array_equal(sel.cpu().numpy(), g[f"{tag}_selected_after"])
    assert float(rec["objective_before"]) == pytest.approx(float(g[f"{tag}_objective_before"]), rel=1e-3)
    assert float(rec["objective_after"]) == pytest.approx(float(g[f"{tag}_objective_after"]), rel=1e-3)
