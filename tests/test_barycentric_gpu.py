"""Control-barycentric two-anchor writer on the GPU
(cast_barycentric_pair_write) against the CPU oracle: bit-exact fp32."""

import numpy as np
import pytest
import torch

from cast_b200 import barycentric
from oracle import barycentric as ob

pytestmark = pytest.mark.gpu


def _case(A, T, S, C, seed):
    g = torch.Generator().manual_seed(seed)
    active = torch.randn(1, A, S, C, generator=g)
    targets = torch.tensor([1, 2, 5, 6], dtype=torch.int32)[: T - 4 if T > 8 else 4]
    pairs = torch.tensor([[0, 1], [0, 1], [2, 3], [3, 4]], dtype=torch.int32)[: targets.numel()]
    weights = torch.softmax(torch.randn(1, targets.numel(), 2, generator=g), dim=-1)
    return active, weights, pairs, targets


@pytest.mark.parametrize("mode", ["fused", "separate", "left_then_right_fma", "right_then_left_fma"])
@pytest.mark.parametrize("S,C", [(880, 64), (7, 5)])
def test_pair_write_matches_oracle(cuda, mode, S, C):
    active, weights, pairs, targets = _case(5, 8, S, C, seed=S + C)
    out = torch.full((1, 8, S, C), 7.0)
    ref = ob.pair_write(active[0].reshape(5, -1).numpy(), weights[0].numpy(), pairs.numpy(),
                        targets.numpy(), out[0].reshape(8, -1).numpy().copy(), ob.MODES[mode])
    got = barycentric.direct_control_barycentric_pair_write(
        active.cuda(), weights.cuda(), pairs.cuda(), targets.cuda(), out.cuda(), arithmetic_mode=mode)
    torch.cuda.synchronize()
    got = got[0].reshape(8, -1).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    # frames that are not targets keep their contents
    assert (got[[0, 3, 4, 7]] == 7.0).all()


def test_pair_write_checks_like_the_reference(cuda):
    active, weights, pairs, targets = _case(3, 8, 7, 5, seed=1)  # 3 anchors: refused
    out = torch.zeros(1, 8, 7, 5, device="cuda")
    with pytest.raises(ValueError, match="4/5/6"):
        barycentric.direct_control_barycentric_pair_write(active.cuda(), weights.cuda(), pairs.cuda(),
                                                          targets.cuda(), out)


def test_pair_write_config4_scale_rate(cuda):
    """Config 4's residual frame (880 x 3072 fp32) with two targets between
    anchors: bit-exact, and the HBM rate (inputs larger than L2)."""
    g = torch.Generator().manual_seed(3)
    active = torch.randn(1, 4, 880, 3072, generator=g).cuda()
    weights = torch.softmax(torch.randn(1, 2, 2, generator=g), dim=-1).cuda()
    pairs = torch.tensor([[0, 1], [0, 1]], dtype=torch.int32).cuda()
    targets = torch.tensor([1, 2], dtype=torch.int32).cuda()
    out = torch.zeros(1, 5, 880, 3072, device="cuda")
    barycentric.direct_control_barycentric_pair_write(active, weights, pairs, targets, out,
                                                      arithmetic_mode="left_then_right_fma")
    torch.cuda.synchronize()
    ref = ob.pair_write(active[0].reshape(4, -1).cpu().numpy(), weights[0].cpu().numpy(),
                        pairs.cpu().numpy(), targets.cpu().numpy(),
                        np.zeros((5, 880 * 3072), np.float32), 2)
    assert np.array_equal(out[0].reshape(5, -1).cpu().numpy().view(np.uint32), ref.view(np.uint32))
    # four input/output sets in turn (4 x 54 MB, more than L2), back to back
    sets = [(torch.randn_like(active), torch.zeros_like(out)) for _ in range(4)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for a_, o_ in sets:
        barycentric.direct_control_barycentric_pair_write(a_, weights, pairs, targets, o_,
                                                          arithmetic_mode="left_then_right_fma")
    # one CUDA graph of 20 launches, so host enqueue time does not show
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for r in range(20):
            a_, o_ = sets[r % 4]
            barycentric.direct_control_barycentric_pair_write(a_, weights, pairs, targets, o_,
                                                              arithmetic_mode="left_then_right_fma")
    graph.replay()
    torch.cuda.synchronize()
    e0.record()
    graph.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / 20
    # algorithmic: the two shared anchor frames read once, two targets written
    nbytes = 4 * 880 * 3072 * 4
    print(f"barycentric pair write (2 targets, 880x3072 fp32): {us:.1f} us, {nbytes / us / 1e3:.0f} GB/s")


def _lift_golden(name):
    import importlib.util
    import os
    here = os.path.join(os.path.dirname(__file__), "golden")
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(here, "make_golden.py"))
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    return mg, np.load(os.path.join(here, f"lift_{name}.npz"))


@pytest.mark.parametrize("name", ["current_only", "memory_boundary", "no_controls", "memory_split"])
def test_lift_matches_reference(cuda, name):
    """The whole control-barycentric lift on the device (weights kernel, then
    the pair writer): the weights within fp32 rounding of the oracle's
    float64 ones, the target rows within 1e-5 of the reference's, the
    anchors copied exactly, the record's counts the reference's."""
    mg, g = _lift_golden(name)
    frames, mem, active, boundary, _, _, lambdas, _ = mg.LIFT_CASES[name]
    act, af, plucker, mouse, keyboard, mm, km = mg.lift_case(name)
    dev = lambda x: None if x is None else x.to(cuda)  # noqa: E731
    full, rec = barycentric.control_barycentric_residual_lift(
        act.to(cuda), af.to(cuda), frames, mem, boundary, plucker.to(cuda), dev(mouse), dev(keyboard),
        dev(mm), dev(km), lambdas, True)
    torch.cuda.synchronize()
    assert rec["targets"] == int(g["n_targets"]) and rec["action_available"] == bool(g["action_available"])
    full = full[0].cpu().numpy()
    np.testing.assert_allclose(full[g["targets"]], g["target_rows"], rtol=0, atol=1e-5)
    assert np.array_equal(full[list(active)], act[0].numpy())
    # the weights kernel alone against the oracle
    npy = lambda x: None if x is None else x[0].float().numpy()  # noqa: E731
    _, w_ref, targets = ob.lift(npy(act), list(active), frames, mem, boundary, npy(plucker), npy(mouse),
                                npy(keyboard), npy(mm), npy(km), lambdas)
    tg = barycentric.lift_targets(list(active), frames, mem, boundary)
    assert [t[:3] for t in tg] == [tuple(t) for t in targets]
    w, _ = barycentric.lift_weights(tg, plucker.to(cuda), dev(mouse), dev(keyboard), dev(mm), dev(km),
                                    total_temporal=frames, memory_temporal=mem, spatial=880,
                                    lambdas=lambdas)
    np.testing.assert_allclose(w[0].cpu().numpy(), w_ref, rtol=0, atol=2e-6)


def test_lift_anchor_only_and_batch_check(cuda):
    """Every frame an anchor: no launch, the residual is the output; batches
    other than 1 are refused."""
    act = torch.randn(1, 4, 880, 16, device=cuda)
    plucker = torch.randn(1, 4 * 880, 6, device=cuda)
    full, rec = barycentric.control_barycentric_residual_lift(
        act, torch.arange(4, device=cuda), 4, 0, None, plucker, None, None, None, None, (1, 1, 1))
    assert rec["targets"] == 0 and rec["direct_pair_kernel_calls"] == 0
    assert torch.equal(full, act)
    with pytest.raises(ValueError, match="batch-1"):
        barycentric.control_barycentric_residual_lift(
            act.expand(2, -1, -1, -1).contiguous(), torch.arange(4, device=cuda), 4, 0, None,
            plucker.expand(2, -1, -1).contiguous(), None, None, None, None, (1, 1, 1))
