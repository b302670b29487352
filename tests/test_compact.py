"""CPU: the compact-path oracle (RoPE phase, rotation, packing, output
scatter) against the fixture made from the reference's own functions."""

import hashlib
import json
import os

import numpy as np
import torch

from cast_b200 import workloads
from oracle import compact as oc

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def oracle_case(tag):
    c = workloads.compact_case(per_head_phase=tag == "heads")
    phase = oc.compact_rope_phase(c.coords.numpy(), c.freqs.numpy(), c.memory_length,
                                  c.memory_latent_idx, c.predict_latent_idx)
    bi, ttp = oc.stable_layout(c.block_id.numpy(), c.n_blocks, c.block_size)
    packed = oc.pack(c.q.float().numpy(), c.k.float().numpy(), c.v.float().numpy(), bi.reshape(-1),
                     phase.real, phase.imag)
    return c, phase, bi, ttp, packed


def test_compact_oracle_matches_reference():
    g = np.load(os.path.join(GOLDEN, "compact_pack.npz"))
    man = json.load(open(os.path.join(GOLDEN, "MANIFEST.json")))["inputs"]
    for tag in ("shared", "heads"):
        c, phase, bi, ttp, packed = oracle_case(tag)
        assert _sha(c.q.view(torch.int16).numpy()) == man[f"compact_{tag}"]["q"]
        ph = np.stack([phase.real, phase.imag], axis=-1).astype(np.float32)
        assert _sha(ph) == str(g[f"{tag}_phase_sha"])
        assert np.array_equal(bi, g[f"{tag}_block_indices"])
        assert np.array_equal(ttp, g[f"{tag}_token_to_packed"])
        assert (bi < 0).any()  # the case has padding slots
        for name, bits in zip("qkv", packed):
            assert _sha(bits.view(np.int16)) == str(g[f"{tag}_{name}_sha"]), (tag, name)
        gen = torch.Generator().manual_seed(11)
        out_packed = torch.randn(tuple(packed[0].shape), generator=gen).bfloat16()
        un = oc.unpack(out_packed.view(torch.int16).numpy(), ttp)
        assert _sha(un) == str(g[f"{tag}_unpack_sha"])
