"""Compact-path packing on the GPU (cast_compact_pack / cast_compact_unpack)
against the CPU oracle: bit-exact bf16 outputs."""

import numpy as np
import pytest
import torch

from cast_b200 import compact, workloads
from oracle import compact as oc

pytestmark = pytest.mark.gpu


def _bits(t):
    return t.detach().cpu().view(torch.int16).numpy().view(np.uint16)


def _layout(c):
    bi, ttp = oc.stable_layout(c.block_id.numpy(), c.n_blocks, c.block_size)
    return bi, ttp


@pytest.mark.parametrize("per_head", [False, True])
@pytest.mark.parametrize("in_dtype", [torch.bfloat16, torch.float32])
def test_pack_matches_oracle(cuda, per_head, in_dtype):
    c = workloads.compact_case(per_head_phase=per_head, heads=3, frames=4)
    phase = oc.compact_rope_phase(c.coords.numpy(), c.freqs.numpy(), c.memory_length,
                                  c.memory_latent_idx, c.predict_latent_idx)
    bi, ttp = _layout(c)
    q, k, v = (t.to(in_dtype) for t in (c.q, c.k, c.v))
    if in_dtype == torch.float32:  # values off the bf16 grid
        q, k = q * 1.001, k * 0.999
    ref = oc.pack(q.float().numpy(), k.float().numpy(), v.float().numpy(), bi.reshape(-1), phase.real, phase.imag)
    out = compact.pack(q.cuda(), k.cuda(), v.cuda(), torch.from_numpy(bi).cuda(),
                       torch.from_numpy(phase).cuda())
    torch.cuda.synchronize()
    for name, o, r in zip("qkv", out, ref):
        assert np.array_equal(_bits(o), r), name
    # no phase: plain gather + cast
    ref0 = oc.pack(q.float().numpy(), k.float().numpy(), v.float().numpy(), bi.reshape(-1))
    out0 = compact.pack(q.cuda(), k.cuda(), v.cuda(), torch.from_numpy(bi).cuda())
    torch.cuda.synchronize()
    for o, r in zip(out0, ref0):
        assert np.array_equal(_bits(o), r)


def test_unpack_inverts_pack(cuda):
    c = workloads.compact_case(heads=4, frames=5)
    bi, ttp = _layout(c)
    qp, kp, vp = compact.pack(c.q.cuda(), c.k.cuda(), c.v.cuda(), torch.from_numpy(bi).cuda())
    back = compact.unpack(vp, torch.from_numpy(ttp).cuda())
    torch.cuda.synchronize()
    assert torch.equal(back.cpu(), c.v)
    ref = oc.unpack(_bits(qp), ttp)
    assert np.array_equal(_bits(compact.unpack(qp, torch.from_numpy(ttp).cuda())), ref)


def test_pack_frame_blocks_large_and_timing(cuda):
    """Config-2 scale (24 heads, 880-token frame blocks of 22x40, 36 frames,
    one memory frame): bit-exact on a sample of rows, unpack round trip, and
    the kernel's HBM rate."""
    c = workloads.compact_case(heads=24, frames=36, hw=(22, 40), cell=(1, 22, 40), seed=9)
    phase = oc.compact_rope_phase(c.coords.numpy(), c.freqs.numpy(), c.memory_length,
                                  c.memory_latent_idx, c.predict_latent_idx)
    bi, ttp = _layout(c)
    qd, kd, vd = c.q.cuda(), c.k.cuda(), c.v.cuda()
    bid, phd = torch.from_numpy(bi).cuda(), torch.from_numpy(phase).cuda()
    out = compact.pack(qd, kd, vd, bid, phd)
    torch.cuda.synchronize()
    flat = bi.reshape(-1)
    rows = np.arange(0, flat.size, 997)
    sub = flat[rows]
    ref = oc.pack(c.q.float().numpy()[:, sub], c.k.float().numpy()[:, sub], c.v.float().numpy()[:, sub],
                  np.arange(sub.size), phase.real[sub], phase.imag[sub])
    for o, r in zip(out, ref):
        assert np.array_equal(_bits(o)[:, :, rows], r)
    assert torch.equal(compact.unpack(out[2], torch.from_numpy(ttp).cuda()).cpu(), c.v)
    # timing: L2 flushed between runs by the inputs' size (3 x 195 MB read)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(3):
        compact.pack(qd, kd, vd, bid, phd, out=out)
    e0.record()
    for _ in range(10):
        compact.pack(qd, kd, vd, bid, phd, out=out)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / 10
    nbytes = 3 * qd.numel() * 2 + 3 * out[0].numel() * 2
    print(f"compact pack L={qd.shape[1]} H=24: {us:.1f} us, {nbytes / us / 1e3:.0f} GB/s")
