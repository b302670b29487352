"""PAR (FC-PASM) parity on the GPU: CUDA kernels vs the reference's own
outputs (golden vectors) and vs the CPU restatement."""

import os

import numpy as np
import pytest
import torch

from cast_b200 import par as cpar
from cast_b200 import workloads
from oracle import par as opar

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
MAX_ABS = 2e-2
MEAN_ABS = 2e-3


def _run_gpu(wl, record_stats=False, tile_confidence=None):
    c = cpar.FCPASMCorrector(record_stats=record_stats)
    c.begin_model_call(chunk_index=1, step_index=0)
    full = wl.full_residual.clone().cuda()
    act = wl.active_residual.cuda()
    out = c.correct(layer_index=5, full_input=None, full_residual=full, active_residual=act,
                    active_frames=torch.tensor(wl.active_frames), memory_length=wl.memory_length,
                    spatial_height=wl.height, spatial_width=wl.width,
                    active_frame_values=tuple(wl.active_frames), tile_confidence=tile_confidence)
    torch.cuda.synchronize()
    assert out.data_ptr() == full.data_ptr()  # in place, as the lean reference path
    return out.cpu(), c


@pytest.mark.parametrize("name,maker", [("par_c64", lambda: workloads.config4(channels=64)),
                                        ("par_motion_c64", lambda: workloads.par_motion(channels=64))])
def test_par_matches_reference_golden(cuda, name, maker):
    wl = maker()
    g = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    out, c = _run_gpu(wl, record_stats=True)
    ref_t = torch.from_numpy(g["targets_bf16_bits"]).view(torch.bfloat16).float()
    got_t = out[0, list(g["target_frames"])].float()
    d = (got_t - ref_t).abs()
    print(f"{name}: vs reference max {float(d.max()):.3e} mean {float(d.mean()):.3e}")
    assert float(d.max()) < MAX_ABS and float(d.mean()) < MEAN_ABS
    assert float(d.max()) < 2e-3  # a few bf16 ulps at this amplitude
    # memory frame untouched, anchors exact copies of active_residual
    assert torch.equal(out[0, 0], wl.full_residual[0, 0])
    for j, f in enumerate(wl.active_frames):
        assert torch.equal(out[0, f], wl.active_residual[0, j])
    st = cpar.unpack_stats(c.last_stats, 1)[0]
    np.testing.assert_allclose(st["base_confidence"].cpu().numpy(), g["stats_base_confidence"], atol=2e-3)
    np.testing.assert_allclose(st["ramp_confidence"].cpu().numpy(), g["stats_ramp_confidence"], atol=2e-3)
    np.testing.assert_allclose(st["displacement"].cpu().numpy(), g["stats_displacement"], atol=2e-3)


def test_par_config4_full_vs_restatement(cuda):
    wl = workloads.config4()
    out, _ = _run_gpu(wl)
    ref = opar.correct(wl.full_residual.float().numpy(), wl.active_residual.float().numpy(),
                       wl.active_frames, wl.memory_length, 22, 40)
    ref_t = torch.from_numpy(ref).to(torch.bfloat16).float()
    d = (out.float() - ref_t).abs()
    print(f"config4 C=3072: max {float(d.max()):.3e} mean {float(d.mean()):.3e}")
    assert float(d.max()) < MAX_ABS and float(d.mean()) < MEAN_ABS
    g = np.load(os.path.join(GOLDEN, "par_cfg4_summary.npz"))
    flat = out[0, [2, 3]].float().reshape(2, -1)
    sample = flat[:, ::int(g["sample_stride"])][:, :4096].numpy()
    assert np.abs(sample - g["sample"]).max() < 2e-3


def _vs_restatement(wl):
    out, _ = _run_gpu(wl)
    ref = opar.correct(wl.full_residual.float().numpy(), wl.active_residual.float().numpy(),
                       wl.active_frames, wl.memory_length, 22, 40)
    ref_t = torch.from_numpy(ref).to(torch.bfloat16).float()
    return (out.float() - ref_t).abs()


@pytest.mark.parametrize("channels", [60, 200])
def test_par_channel_edges(cuda, channels):
    """C = 60 (C % 8 != 0) takes the per-channel DFT kernels; C = 200 the
    tensor-core kernels with a ragged second 128-channel chunk (zero-filled
    loads, masked stores)."""
    d = _vs_restatement(workloads.config4(channels=channels))
    print(f"C={channels}: max {float(d.max()):.3e} mean {float(d.mean()):.3e}")
    assert float(d.max()) < 2e-3 and float(d.mean()) < MEAN_ABS


def test_par_two_anchor_pairs(cuda):
    """One memory frame, anchors at current frames 0, 3 | 4, 7 (the segment
    boundary is 4): pairs (0, 3) with targets 1, 2 and (4, 7) with targets
    5, 6 -- two pairs' statistics and four targets' F images and predicted
    tiles in the persistent kernels' orderings; C = 136 leaves an 8-channel
    second chunk."""
    g = torch.Generator().manual_seed(11)
    full = (torch.randn(1, 9, 880, 136, generator=g) * 0.02).to(torch.bfloat16)
    wl = workloads.PARWorkload("two_pairs", full, [0, 1, 4, 5, 8], 1, 22, 40)
    d = _vs_restatement(wl)
    print(f"two pairs: max {float(d.max()):.3e} mean {float(d.mean()):.3e}")
    assert float(d.max()) < 2e-3 and float(d.mean()) < MEAN_ABS


def test_par_injected_confidence_exercises_phase(cuda):
    """Config 4's c~U(0,1) mode: per-tile confidence injected (the reference's
    precomputed_tile_confidence), g from the same sigmoid; compared with the
    restatement given the same confidence."""
    wl = workloads.config4(channels=256)
    conf = torch.rand(1, 18, generator=torch.Generator().manual_seed(4))
    out, _ = _run_gpu(wl, tile_confidence=conf)
    pairs_conf = {(0, 3): conf[0].double().numpy()}
    ref = opar.correct(wl.full_residual.float().numpy(), wl.active_residual.float().numpy(),
                       wl.active_frames, wl.memory_length, 22, 40, tile_confidence=pairs_conf)
    ref_t = torch.from_numpy(ref).to(torch.bfloat16).float()
    d = (out.float() - ref_t).abs()
    assert float(d.max()) < 2e-3


def test_par_fallbacks_leave_residual(cuda):
    wl = workloads.config4(channels=64)
    c = cpar.FCPASMCorrector()
    c.begin_model_call(chunk_index=0, step_index=0)
    full = wl.full_residual.clone().cuda()
    out = c.correct(layer_index=1, full_input=None, full_residual=full, active_residual=wl.active_residual.cuda(),
                    active_frames=torch.tensor(wl.active_frames), memory_length=1, spatial_height=22,
                    spatial_width=40, active_frame_values=tuple(wl.active_frames))
    assert torch.equal(out.cpu(), wl.full_residual) and c._records[-1]["fallback_reason"] == "first_chunk"
