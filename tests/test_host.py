"""CPU: the C-ABI library loads, exports every declared symbol, and its host
validation fails closed (no device work is issued by these calls)."""

import ctypes
import os
import re

import pytest

from cast_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "cast_b200.h")


def _declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(cast_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from cast_b200 import build

    build.build()
    return _lib.load()


def test_every_declared_symbol_is_exported_and_bound(lib):
    names = _declared()
    assert len(names) >= 10
    for n in names:
        assert hasattr(lib, n), n
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"


def test_status_strings(lib):
    assert lib.cast_status_string(0) == b"CAST_OK"
    assert lib.cast_status_string(3) == b"CAST_ERR_ALIGNMENT"
    assert lib.cast_version() >= 100


def test_attention_rejects_null_and_unsupported(lib):
    st = lib.cast_rcsa_attention(*([None] * 10), 1, None, 1, 1, 128, 128, 128, 128, 128, 0.1,
                                 None, None, None, None, 0, None)
    assert st == 1 and b"required" in lib.cast_last_error_message()
    fake = ctypes.c_void_p(4096)
    st = lib.cast_rcsa_attention(fake, fake, fake, None, None, None, None, None, fake, fake, 1, None,
                                 1, 1, 128, 128, 64, 128, 128, 0.1, fake, None, None, None, 0, None)
    assert st == 2 and b"head_dim" in lib.cast_last_error_message()
    st = lib.cast_rcsa_attention(fake, fake, fake, None, None, None, None, None, fake, fake, 300, None,
                                 1, 1, 128, 128, 128, 110, 110, 0.1, fake, None, None, None, 0, None)
    assert st == 2 and b"max_degree 300" in lib.cast_last_error_message()
    odd = ctypes.c_void_p(4097)
    st = lib.cast_rcsa_attention(odd, fake, fake, None, None, None, None, None, fake, fake, 1, None,
                                 1, 1, 128, 128, 128, 128, 128, 0.1, fake, None, None, None, 0, None)
    assert st == 3


def test_select_quant_validation(lib):
    fake = ctypes.c_void_p(4096)
    args = [fake, fake, None, None, None, 1, 1, 880, 1760, 128, 880, 8, 0, fake, fake] + [None] * 6 + [fake]
    st = lib.cast_rcsa_select_quant(*args, 2, 0.025, None, None, 0, None)
    assert st == 1  # auto policy with a qk_mode output needs code buffers
    args2 = [fake, fake, None, None, None, 1, 1, 880, 1760, 96, 880, 8, 0, fake, fake] + [None] * 7
    st = lib.cast_rcsa_select_quant(*args2, 0, 0.025, None, None, 0, None)
    assert st == 2
    need = lib.cast_rcsa_select_quant_workspace_bytes(1, 24, 3520, 31680, 128, 880)
    assert need >= 24 * 40 * 128 * 8
    st = lib.cast_rcsa_select_quant(*args[:-7], *([None] * 7), 0, 0.025, None, fake, 16, None)
    assert st == 4 and b"workspace" in lib.cast_last_error_message()


def test_par_validation(lib):
    frames = (ctypes.c_int32 * 3)(0, 3, 1)
    fake = ctypes.c_void_p(4096)
    st = lib.cast_par_fcpasm(fake, fake, ctypes.cast(frames, ctypes.c_void_p), 3, 5, 1, 22, 40, 64,
                             0.5, 0.75, 2.0, 0.03, 1, 4, None, None, fake, 1 << 30, None)
    assert st == 1 and b"sorted" in lib.cast_last_error_message()
    st = lib.cast_par_fcpasm(fake, fake, ctypes.cast(frames, ctypes.c_void_p), 3, 5, 1, 24, 40, 64,
                             0.5, 0.75, 2.0, 0.03, 1, 4, None, None, fake, 1 << 30, None)
    assert st == 2


def test_python_wrappers_refuse_cpu_tensors():
    import torch

    from cast_b200 import rcsa

    q = torch.zeros(1, 1, 128, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        rcsa.select_quant(q, q, block_size=128, budget=1)


def test_compact_and_pair_writer_validation(lib):
    fake = ctypes.c_void_p(4096)
    # compact packing: head_dim other than 128, bad dtype code, bad phase heads
    st = lib.cast_compact_pack(fake, fake, fake, 0, None, 1, fake, 1, 8, 2, 64, 8, fake, fake, fake, None)
    assert st == 2 and b"head_dim" in lib.cast_last_error_message()
    st = lib.cast_compact_pack(fake, fake, fake, 7, None, 1, fake, 1, 8, 2, 128, 8, fake, fake, fake, None)
    assert st == 1 and b"in_dtype" in lib.cast_last_error_message()
    st = lib.cast_compact_pack(fake, fake, fake, 0, fake, 3, fake, 1, 8, 2, 128, 8, fake, fake, fake, None)
    assert st == 1 and b"phase_heads" in lib.cast_last_error_message()
    st = lib.cast_compact_unpack(None, fake, 1, 8, 2, 128, 8, fake, None)
    assert st == 1
    # pair writer: unknown arithmetic mode, misaligned frames
    st = lib.cast_barycentric_pair_write(fake, fake, fake, fake, fake, 4, 5, 2, 880 * 64, 9, None)
    assert st == 1 and b"arithmetic_mode" in lib.cast_last_error_message()
    odd = ctypes.c_void_p(4097)
    st = lib.cast_barycentric_pair_write(odd, fake, fake, fake, fake, 4, 5, 2, 880 * 64, 2, None)
    assert st == 3


def test_pair_writer_wrapper_checks_like_the_reference():
    import torch

    from cast_b200 import barycentric

    act = torch.zeros(1, 4, 8, 4)
    with pytest.raises(ValueError, match="CUDA"):
        barycentric.direct_control_barycentric_pair_write(
            act, torch.zeros(1, 2, 2), torch.zeros(2, 2, dtype=torch.int32),
            torch.zeros(2, dtype=torch.int32), torch.zeros(1, 5, 8, 4))


def test_compact_wrapper_refuses_cpu_tensors():
    import torch

    from cast_b200 import compact

    x = torch.zeros(1, 8, 2, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        compact.pack(x, x, x, torch.zeros(8, dtype=torch.int32))


def test_host_plan_value_runs():
    """The selected-values copy plan: per head, the union of the selected
    blocks (entries past a row's count and outside [0, nkb) ignored), runs
    of consecutive blocks merged, and runs at most ``value_gap`` blocks apart
    merged across the gap; the ragged last block ends at Lk."""
    import torch

    from cast_b200 import rcsa

    hp = object.__new__(rcsa.RCSAHostPlan)
    hp.shape = (1, 2, 1760, 10 * 100 - 40, 128)  # Lk = 960: 10 blocks of 100, the last ragged
    hp.block_size = 100
    hp.heads = [(4, 6)]
    idx = torch.full((1, 2, 2, 6), -1, dtype=torch.int32)
    idx[0, 0, 0, :4] = torch.tensor([3, 4, 7, 9])
    idx[0, 0, 1, :5] = torch.tensor([0, 4, 12, -1, 9])  # 12 is out of range, -1 skipped
    idx[0, 1, 0, :2] = torch.tensor([5, 2])
    idx[0, 1, 1, :6] = torch.tensor([6, 6, 1, 8, 8, 8])  # only the first 3 counted
    cnt = torch.tensor([[[4, 5], [2, 3]]], dtype=torch.int32)
    hp._sel_host = [(idx, cnt)]
    hp.value_gap = 0
    assert hp._value_runs(0) == [(4, 0, 100), (4, 300, 500), (4, 700, 800), (4, 900, 960),
                                 (5, 100, 300), (5, 500, 700)]
    hp.value_gap = 1
    assert hp._value_runs(0) == [(4, 0, 100), (4, 300, 500), (4, 700, 960), (5, 100, 300), (5, 500, 700)]
    hp.value_gap = 2
    assert hp._value_runs(0) == [(4, 0, 960), (5, 100, 700)]
