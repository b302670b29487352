"""cast_rcsa_select_quant_noalloc: the allocation-free selection entry point.

It must give exactly the results of cast_rcsa_select_quant (which takes a
caller workspace) while using the library's static scratch.  Two calls are
enqueued back to back on one stream before anything is read, so the second
reuses scratch the first left behind.  This file is named to be collected
last, so it also runs after every other test has used the device.
"""

import ctypes

import pytest
import torch

from cast_b200 import _lib, rcsa

CAST_ERR_WORKSPACE = 4
NOALLOC_SCRATCH_BYTES = 8 << 20  # CAST_NOALLOC_SCRATCH_BYTES in include/cast_b200.h


def _problem(b, h, lq, lk, d, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, h, lq, d, generator=g).bfloat16()
    k = torch.randn(b, h, lk, d, generator=g).bfloat16()
    v = torch.randn(b, h, lk, d, generator=g).bfloat16()
    return q, k, v


def _outputs(q, k, v, block, budget):
    b, h, lq, d = q.shape
    lk = k.shape[2]
    nqb, nkb = -(-lq // block), -(-lk // block)
    deg = min(budget, nkb - nqb) + nqb
    dev = q.device
    return dict(
        idx=torch.full((b, h, nqb, deg), -7, dtype=torch.int32, device=dev),
        cnt=torch.full((b, h, nqb), -7, dtype=torch.int32, device=dev),
        qc=torch.zeros(b, h, lq, d, dtype=torch.int8, device=dev),
        qs=torch.zeros(b, h, nqb, dtype=torch.float32, device=dev),
        kc=torch.zeros(b, h, lk, d, dtype=torch.int8, device=dev),
        ks=torch.zeros(b, h, nkb, dtype=torch.float32, device=dev),
        vc=torch.zeros(b, h, lk, d, dtype=torch.int8, device=dev),
        vs=torch.zeros(b, h, nkb, dtype=torch.float32, device=dev),
        mode=torch.full((b, h, nqb), 9, dtype=torch.uint8, device=dev),
        pooled=torch.zeros(b, h, nqb + nkb, d, dtype=torch.float64, device=dev),
    )


def _args(q, k, v, block, budget, o):
    b, h, lq, d = q.shape
    P = _lib.ptr
    return [P(q), P(k), P(v), None, None, b, h, lq, k.shape[2], d, block, budget, rcsa.RULE_BUDGET_CAUSAL,
            P(o["idx"]), P(o["cnt"]), P(o["qc"]), P(o["qs"]), P(o["kc"]), P(o["ks"]), P(o["vc"]),
            P(o["vs"]), P(o["mode"]), rcsa.POLICIES["auto"], 0.025, P(o["pooled"])]


def _stream():
    return torch.cuda.current_stream().cuda_stream


CASES = [
    # (b, h, lq, lk, d, block, budget, seed); the second reuses the first's scratch
    (1, 3, 512, 2048, 128, 64, 8, 1),
    (2, 2, 200, 1000, 64, 32, 5, 2),
]


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point(cuda):
    lib = _lib.load()
    problems, got = [], []
    for b, h, lq, lk, d, block, budget, seed in CASES:
        q, k, v = (t.to(cuda) for t in _problem(b, h, lq, lk, d, seed))
        assert lib.cast_rcsa_select_quant_workspace_bytes(b, h, lq, lk, d, block) <= NOALLOC_SCRATCH_BYTES
        o = _outputs(q, k, v, block, budget)
        _lib.call("cast_rcsa_select_quant_noalloc", *_args(q, k, v, block, budget, o), _stream())
        problems.append((q, k, v, block, budget))
        got.append(o)
    torch.cuda.synchronize()
    assert lib.cast_device_error(_stream()) == 0

    for (q, k, v, block, budget), o in zip(problems, got):
        ref = _outputs(q, k, v, block, budget)
        b, h, lq, d = q.shape
        nbytes = lib.cast_rcsa_select_quant_workspace_bytes(b, h, lq, k.shape[2], d, block)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=cuda)
        _lib.call("cast_rcsa_select_quant", *_args(q, k, v, block, budget, ref), _lib.ptr(ws),
                  nbytes, _stream())
        torch.cuda.synchronize()
        for name in ref:
            assert torch.equal(o[name], ref[name]), f"{name} differs for shape {tuple(q.shape)}"
        assert (o["cnt"] > 0).all()


def test_noalloc_rejects_oversize_before_launch():
    """Sizes whose scratch exceeds the static array fail on the host, with no
    device work (so this runs without a GPU too)."""
    lib = _lib.load()
    b, h, lq, lk, d, block = 1, 64, 4096, 65536, 128, 64
    need = lib.cast_rcsa_select_quant_workspace_bytes(b, h, lq, lk, d, block)
    assert need > NOALLOC_SCRATCH_BYTES
    args = [None, None, None, None, None, b, h, lq, lk, d, block, 16, 0] + [None] * 9 + [2, 0.025, None, None]
    status = lib.cast_rcsa_select_quant_noalloc(*args)
    assert status == CAST_ERR_WORKSPACE
    msg = lib.cast_last_error_message().decode()
    assert "static scratch" in msg and str(need) in msg
