"""The compact CWCA attention on the B200 (``cast_compact_select`` and the
frame weave's ``_compact_cwca_attention`` replacement) against the oracle and
against the selection the reference's own method produced on the same layout
(``tests/golden/compact_select_*.npz``)."""

import os
import types

import numpy as np
import pytest
import torch

from cast_b200 import compact, compact_attention
from oracle import rcsa as orc
from test_oracle_golden import assert_same_rows

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
MAX_ABS, MEAN_ABS = 2e-2, 2e-3
CASES = ["uniform", "curved", "tt2"]


def _mg():
    import importlib.util

    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLDEN, "make_golden.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


MG = _mg()


def _case(name):
    frames, mem, active, shape, heads, curvature, _ = MG.COMPACT_SELECT_CASES[name]
    q, k, v = MG.compact_select_case(name)
    g = np.load(os.path.join(GOLDEN, f"compact_select_{name}.npz"))
    tt, th, tw = shape
    nh, nw = -(-22 // th), -(-40 // tw)
    cells = g["block_indices"].shape[0] // (nh * nw)
    return dict(frames=frames, mem=mem, active=active, shape=shape, curvature=curvature, q=q, k=k, v=v,
                g=g, grid=(cells, nh, nw))


@pytest.mark.parametrize("policy", ["bf16", "auto", "int8"])
@pytest.mark.parametrize("name", CASES)
def test_compact_select_kernel(cuda, name, policy):
    c = _case(name)
    g = c["g"]
    bi = torch.from_numpy(g["block_indices"])
    block = bi.shape[1]
    qp, kp, vp = compact.pack(c["q"].cuda(), c["k"].cuda(), c["v"].cuda(), bi.cuda())
    degrees = torch.from_numpy(g["counts"][0, 0])
    idx, cnt, qc, qs, kc, ks, mode = compact_attention.compact_select(
        qp, kp, torch.from_numpy(g["valid"]).cuda(), degrees, block_size=block, grid=c["grid"][1:],
        policy=policy)
    torch.cuda.synchronize()
    qpn, kpn = (orc.compact_pack(t.float().numpy(), g["block_indices"]) for t in (c["q"], c["k"]))
    valid = g["valid"].reshape(-1)
    sel, ocnt, _ = orc.compact_select(qpn, kpn, valid, block, c["grid"], degrees.numpy())
    np.testing.assert_array_equal(idx.cpu().numpy(), sel)     # the oracle's order, ties included
    np.testing.assert_array_equal(cnt.cpu().numpy(), ocnt)
    assert_same_rows(idx.cpu().numpy(), g["selected"], ocnt)   # the reference's blocks
    if policy == "int8":
        codes, scales = orc.quantize_blocks(qpn, block, valid.astype(bool))
        np.testing.assert_array_equal(qs.cpu().numpy(), scales)
        np.testing.assert_array_equal(qc.cpu().numpy(), codes)
        assert bool(mode.all())


def _weave_and_layout(c):
    g = c["g"]
    tt = c["shape"][0]
    weave = types.SimpleNamespace(
        geometry_provider=types.SimpleNamespace(mode="open_loop"), sparse_density=0.2,
        _current_curvature=(lambda n, cv=c["curvature"]: None if cv is None
                            else torch.tensor(cv, dtype=torch.float32)[:n]),
        fc_pasm_swap_router=None, world_spectral_corrector=None, routing_mode="fc_pasm_swap",
        routing_skip_inactive_layers=True)
    layout = types.SimpleNamespace(
        compact_block_indices=torch.from_numpy(g["block_indices"]).cuda(),
        compact_block_valid=torch.from_numpy(g["valid"]).cuda(),
        compact_token_to_packed=torch.from_numpy(g["token_to_packed"]).cuda(),
        compact_block_shape=c["shape"], packed_block_size=int(g["block_indices"].shape[1]),
        spatial_height=22, spatial_width=40, active_frame_values=tuple(c["active"]),
        memory_temporal=c["mem"], active_frames=torch.tensor(c["active"]).cuda(),
        total_temporal=c["frames"])
    del tt
    return weave, layout


@pytest.mark.parametrize("policy", ["bf16", "auto"])
@pytest.mark.parametrize("name", CASES)
def test_compact_cwca_attention_matches_oracle(cuda, name, policy):
    """The whole replaced method: packing, degrees, ranking, attention with
    the policy's precision, scatter back to token order -- against the
    oracle's explicit softmax over the reference's selection."""
    c = _case(name)
    g = c["g"]
    weave, layout = _weave_and_layout(c)

    def refuse(*a, **k):
        raise AssertionError("the reference method must not run for CUDA tensors here")

    module = types.SimpleNamespace(block_idx=5, o=lambda t: t)
    out = compact_attention.compact_cwca_attention(weave, module, c["q"].cuda(), c["k"].cuda(),
                                                   c["v"].cuda(), layout, original=refuse, policy=policy)
    torch.cuda.synchronize()
    rec = weave._last_compact_attention
    assert rec["edge_budget"] == int(g["edge_budget"]) and rec["maximum_degree"] == int(g["maximum_degree"])
    bi = g["block_indices"]
    qp, kp, vp = (orc.compact_pack(t.float().numpy(), bi) for t in (c["q"], c["k"], c["v"]))
    ref = orc.block_sparse_attention(qp, kp, vp, g["selected"], g["counts"], bi.shape[1], bi.shape[1],
                                     key_valid=g["valid"].reshape(-1).astype(bool))
    ttp = g["token_to_packed"]
    ref_tok = np.transpose(ref[:, :, ttp], (0, 2, 1, 3)).reshape(out.shape)
    d = np.abs(out.float().cpu().numpy() - ref_tok)
    print(f"{name} {policy}: max {d.max():.3e} mean {d.mean():.3e}")
    assert d.max() < MAX_ABS and d.mean() < MEAN_ABS
