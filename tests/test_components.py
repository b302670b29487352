"""CPU: the drop-in against the reference package itself.

``cast_b200.make_cast_components()`` must patch every seam it claims on the
reference's own factory triple, keep the reference's code for host tensors
and unsupported FC knobs, and hand the reference corrector's routing cache to
the B200 corrector.  These tests import the reference package from the source
tree given by ``CAST_REFERENCE_SRC`` (default: the survey location); where it
is absent (the GPU box) they skip.
"""

import importlib
import importlib.util
import os
import sys

import numpy as np
import pytest
import torch

from cast_b200 import components, par, workloads

REF_SRC = os.environ.get("CAST_REFERENCE_SRC", "/root/reference/src")


@pytest.fixture(scope="module")
def factory():
    if not os.path.isdir(os.path.join(REF_SRC, "interaction_accel")):
        pytest.skip("the CAST reference package is not present")
    if REF_SRC not in sys.path:
        sys.path.insert(0, REF_SRC)
    saved = torch.cuda.current_stream
    # the reference's PAR path asks for the current stream (proposed/
    # matrix_world_spectral_residual.py:3007); on a CPU-only host it is a no-op
    torch.cuda.current_stream = lambda *a, **k: None
    yield importlib.import_module("interaction_accel.cast_matrix")
    torch.cuda.current_stream = saved
    components.uninstall_kernels()


def test_every_claimed_seam_is_patched(factory):
    memory, attention, weave = components.make_cast_components()
    seams = components.patched_seams(weave)
    assert seams == {k: True for k in seams}, seams
    assert set(seams) == {"longcat_active", "longcat_asymmetric", "pair_write", "taba_select",
                          "compact_cwca", "lift", "correct", "refine"}
    # the attention compiler reaches the patched TABA select through super()
    qk = importlib.import_module("interaction_accel.methods.proposed.qk_uncertainty_tangent_attention")
    assert isinstance(attention, qk.MatrixTrajectoryAdaptiveBudgetAttentionCompiler)
    # the factory's corrector runs the FC-PASM path the kernels implement
    ref = weave.world_spectral_corrector
    assert components.unsupported_fc_knob(ref) is None
    assert ref._fc_routing_publish_layers == frozenset({21, 25})
    # installing twice patches once
    components.install_kernels()
    components.attach(weave)
    assert components.patched_seams(weave) == seams


def test_uninstall_restores_reference_seams(factory):
    components.install_kernels()
    components.uninstall_kernels()
    seams = components.patched_seams()
    assert not any(seams.values()), seams
    components.install_kernels()
    assert all(components.patched_seams().values())


def test_host_tensors_keep_reference_lift(factory):
    """CPU residuals run the reference's own control-barycentric lift through
    the patched classmethod: the same rows as the golden."""
    components.make_cast_components()
    weave_mod = importlib.import_module("interaction_accel.methods.proposed.matrix_curvature_phase_frame_weave")
    spec = importlib.util.spec_from_file_location(
        "make_golden", os.path.join(os.path.dirname(__file__), "golden", "make_golden.py"))
    gold = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gold)
    act, af, plucker, mouse, keyboard, mm, km = gold.lift_case("memory_boundary")
    frames, mem, _, boundary, _, _, lambdas, _ = gold.LIFT_CASES["memory_boundary"]
    full, rec = weave_mod.MatrixCurvaturePhaseFrameWeave._control_barycentric_residual_lift(
        act, af, frames, mem, boundary, plucker, mouse, keyboard, mm, km, lambdas, True)
    assert "backend" not in rec
    ref = np.load(os.path.join(os.path.dirname(gold.__file__), "lift_memory_boundary.npz"))
    assert np.array_equal(full[0, ref["targets"]].numpy(), ref["target_rows"])


def test_host_tensors_keep_reference_correct(factory):
    """CPU residuals run the reference's own correct(); the call is counted."""
    _, _, weave = components.make_cast_components()
    ref = weave.world_spectral_corrector
    ref.begin_model_call(geometry=None, chunk_index=1, step_index=0, device=torch.device("cpu"))
    ref.fc_triton_tile_extract = False   # the Triton extractor needs a GPU
    wl = workloads.par_motion(channels=64)
    full = wl.full_residual.clone()
    ref.correct(layer_index=21, full_input=full, full_residual=full, active_residual=wl.active_residual,
                active_frames=torch.tensor(wl.active_frames), memory_length=1, spatial_height=22,
                spatial_width=40, active_frame_values=tuple(wl.active_frames))
    assert ref._cast_b200_reference_calls == {"host_tensors": 1}
    assert ref._records[-1]["status"] == "corrected"
    # the reference published for its router at layer 22
    assert ref.fc_pasm_routing_transport(layer_index=22) is not None


def test_unsupported_knobs_are_named(factory):
    _, _, weave = components.make_cast_components()
    ref = weave.world_spectral_corrector
    saved = ref.fc_transport_tile_topk
    try:
        ref.fc_transport_tile_topk = 3
        assert components.unsupported_fc_knob(ref) == "fc_transport_tile_topk"
    finally:
        ref.fc_transport_tile_topk = saved


def test_taba_select_host_tensors_are_the_reference(factory):
    """CPU tensors through the patched class method give the reference's own
    selection (the CUDA path is compared in the GPU tests)."""
    qk = importlib.import_module("interaction_accel.methods.proposed.qk_uncertainty_tangent_attention")
    components.install_kernels()
    cls = qk.MatrixTrajectoryAdaptiveBudgetAttentionCompiler
    assert cls.select is components._taba_select
    called = []
    orig = components._PATCHED["taba_select"]
    components._PATCHED["taba_select"] = lambda *a, **k: called.append(1) or orig(*a, **k)
    try:
        comp = type("C", (), {"_row_degrees": None})()
        with pytest.raises(RuntimeError, match="not compiled"):
            components._taba_select(comp, torch.zeros(1, 1, 4, 8), torch.zeros(1, 1, 4, 8),
                                    geometry_indices=None, geometry_counts=None, latent_hw=(2, 2),
                                    block_shape=(1, 1, 1))
        assert called == [1]
    finally:
        components._PATCHED["taba_select"] = orig


def test_shared_routing_cache(factory):
    """The B200 corrector writes into the reference corrector's own cache
    (the dict the weave's fc_pasm_routing_transport reads)."""
    _, _, weave = components.make_cast_components()
    ref = weave.world_spectral_corrector
    cache = ref._fc_routing_transport
    ref.begin_model_call(geometry=None, chunk_index=1, step_index=2, device=torch.device("cpu"))
    assert ref._fc_routing_transport is cache   # cleared in place
    fake = {"pairs": {}}
    cache[(2, 21)] = fake
    assert ref.fc_pasm_routing_transport(layer_index=22) is fake


@pytest.mark.parametrize("anchors,length,boundary,targets,pairs", [
    ([0, 3], 4, 4, [1, 2], [(0, 3)]),
    ([0, 3, 4, 7], 8, 4, [1, 2, 5, 6], [(0, 3), (4, 7)]),
    ([0, 2, 3], 4, 4, [1], [(0, 2)]),
    ([0, 5], 6, 4, [], []),              # anchors in different segments never pair
    # 3 | 6 straddle the boundary: frames 4, 5 have no left anchor in their
    # segment, frames 0 and 7 no bracket at all
    ([1, 3, 6], 8, 4, [2], [(1, 3)]),
])
def test_bracket_rule(anchors, length, boundary, targets, pairs):
    t, _, p = par.bracket_targets(anchors, length, boundary)
    assert t == targets and p == pairs


def test_bracket_rule_matches_reference_records(factory):
    """The reference corrector's own record of targets and pairs (lean
    reference-numerics path, :3672-3690) for several anchor layouts."""
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
    import make_golden as mg

    g = torch.Generator().manual_seed(3)
    for active, mem in (([0, 1, 4], 1), ([0, 1, 4, 5, 8], 1), ([0, 1, 3, 4], 1), ([0, 2, 5, 6], 1)):
        frames = max(active) + 1
        full = (torch.randn(1, frames, 880, 16, generator=g) * 0.02).to(torch.bfloat16)
        wl = workloads.PARWorkload("b", full, active, mem, 22, 40)
        c = mg.par_corrector()
        c.correct(layer_index=3, full_input=full, full_residual=full.clone(),
                  active_residual=wl.active_residual, active_frames=torch.tensor(active),
                  memory_length=mem, spatial_height=22, spatial_width=40,
                  active_frame_values=tuple(active))
        rec = c._records[-1]
        anchors = [f - mem for f in active if f >= mem]
        t, pot, p = par.bracket_targets(anchors, frames - mem, 4)
        if rec["status"] != "corrected":
            assert t == []
            continue
        assert t == list(rec["target_frames"])
        assert [list(p[i]) for i in pot] == [list(x) for x in rec["target_anchor_pairs"]]


def test_transport_goldens_are_self_consistent():
    """The committed layer-21 -> 22 fixtures: the published pairs are the
    bracket rule's, and the routers refined on them."""
    here = os.path.join(os.path.dirname(__file__), "golden")
    for name, anchors, length in (("one_pair", [0, 3], 4), ("two_pairs", [0, 3, 4, 7], 8)):
        g = np.load(os.path.join(here, f"transport_{name}.npz"))
        _, _, p = par.bracket_targets(anchors, length, 4)
        assert [tuple(x) for x in g["pairs"]] == p
        assert list(g["exact_frames"]) == anchors
        for tag in ("production", "two_rounds"):
            assert str(g[f"{tag}_status"]) == "refined" and int(g[f"{tag}_swap_count"]) >= 1


def _golden_module():
    import importlib.util
    here = os.path.join(os.path.dirname(__file__), "golden")
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(here, "make_golden.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("name", ["uniform", "curved", "tt2"])
def test_compact_degrees_match_reference(factory, name):
    """The host-side degree split of the B200 compact path equals the counts
    the reference's ``_compact_cwca_attention`` handed to its attention launch
    (tests/golden/compact_select_*.npz), on the reference's own weave and
    layout."""
    import types

    from cast_b200 import compact_attention as ca

    mg = _golden_module()
    frames, mem, active, shape, heads, curvature, _ = mg.COMPACT_SELECT_CASES[name]
    _, _, weave = components.make_cast_components()
    weave.geometry_provider = types.SimpleNamespace(mode="open_loop")
    weave._current_curvature = (lambda n, c=curvature: None if c is None
                                else torch.tensor(c, dtype=torch.float32)[:n])
    layout = weave._layout(x=torch.zeros(1, frames * 880, 8), grid_sizes=torch.tensor([[frames, 22, 40]]),
                           memory_length=mem, active_frames=torch.tensor(active),
                           orbit_sparse_layout=types.SimpleNamespace(block_shape=shape))
    tt, th, tw = shape
    nh, nw = -(-22 // th), -(-40 // tw)
    blocks = layout.compact_block_indices.shape[0]
    cells = blocks // (nh * nw)
    memory_frames = sum(1 for f in active if f < mem)
    deg, _, meta = ca.compact_degrees(weave, layout, layer_index=5, blocks=blocks,
                                      local_max=ca.stencil_max(cells, nh, nw), spatial=nh * nw, tt=tt,
                                      compact_frames=len(active), memory_frames=memory_frames,
                                      provider=None, device=torch.device("cpu"))
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", f"compact_select_{name}.npz"))
    np.testing.assert_array_equal(deg.numpy(), g["counts"][0, 0])
    assert meta is None
    # the stencil maximum the reference computes with a [blocks, blocks] mask
    ids = torch.arange(blocks)
    bt, rem = ids // (nh * nw), ids % (nh * nw)
    local = ((bt[:, None] - bt[None]).abs() + (rem // nw)[:, None].sub((rem // nw)[None]).abs()
             + (rem % nw)[:, None].sub((rem % nw)[None]).abs()) <= 1
    assert ca.stencil_max(cells, nh, nw) == int(local.sum(-1).max())


def test_compact_degrees_closed_loop_provider_is_consulted():
    """With a closed-loop provider the current rows' degrees are the
    provider's, as the reference takes them (:5754-5772)."""
    import types

    from cast_b200 import compact_attention as ca

    calls = {}

    class Provider:
        mode = "closed_loop"

        def compact_closed_loop_degrees(self, **kw):
            calls.update(kw)
            n = kw["total_blocks"] - kw["memory_blocks"]
            return torch.arange(n) % 3 + kw["base_degree"], {"source": "fake", "previous_layer": 4}

    layout = types.SimpleNamespace(active_frames=torch.tensor([0, 2, 3]), memory_temporal=1,
                                   total_temporal=4)
    weave = types.SimpleNamespace(sparse_density=0.5)
    deg, mean, meta = ca.compact_degrees(weave, layout, layer_index=7, blocks=12, local_max=4, spatial=4,
                                         tt=1, compact_frames=3, memory_frames=1, provider=Provider(),
                                         device=torch.device("cpu"))
    assert mean == 6 and meta["source"] == "fake" and calls["layer_index"] == 7
    assert calls["base_degree"] == 5 and calls["memory_blocks"] == 4
    assert int(deg.sum()) == 12 * 6 and int(deg.max()) <= 12
