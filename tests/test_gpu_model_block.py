"""kv_execution="packed" at the model level: one transformer block's forward over a packed past.

The reference (``make_golden.py``) ran ``DiffusionTransformerBlock._compute_block`` with the past
from its own ``PackedKVCache`` (pack -> unpack, the packed backend's path) and recorded the
block's hidden output, its own K/V and the attention output.  Here the same block (same seeded
parameters, same attribute names) runs through ``packed_block_forward``: the projections and the
FFN as torch modules, the attention over the packed past plus this step's K/V in the kernels.
Attention output within relative L2 1e-3; hidden output and K/V within the same bound.
"""

import numpy as np
import pytest
import torch
import torch.nn as nn

from golden_lib import BLOCK_PARAM_ORDER, array_digest, block_params, case_arrays, load_pins

pytestmark = pytest.mark.gpu

REL_L2_TOL = 1e-3


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


class Block(nn.Module):
    """The module layout of shadowinfer/models/simple_diffusion_llm.py:26-52 (attribute names,
    shapes), filled with the fixture's seeded parameters."""

    def __init__(self, H, D, inter, params):
        super().__init__()
        hidden = H * D
        self.hidden_dim, self.num_heads, self.head_dim = hidden, H, D
        self.ln1 = nn.LayerNorm(hidden)
        self.q_proj = nn.Linear(hidden, hidden)
        self.k_proj = nn.Linear(hidden, hidden)
        self.v_proj = nn.Linear(hidden, hidden)
        self.o_proj = nn.Linear(hidden, hidden)
        self.ln2 = nn.LayerNorm(hidden)
        self.up_proj = nn.Linear(hidden, inter)
        self.down_proj = nn.Linear(inter, hidden)
        with torch.no_grad():
            named = dict(self.named_parameters())
            for name in BLOCK_PARAM_ORDER:
                named[name].copy_(params[name])


@pytest.fixture(scope="module")
def skv():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import shadow_infer_b200.shadowkv as m
    return m


@pytest.mark.parametrize("case", sorted(c for c, v in load_pins()["cases"].items() if v["kind"] == "block"))
def test_block_forward_over_packed_past(case, skv, golden_small, golden_pins):
    pin = golden_pins["cases"][case]
    a = case_arrays(golden_small, case)
    params = block_params(pin["seed"], pin["H"] * pin["D"], pin["inter"])
    assert {n: array_digest(params[n]) for n in BLOCK_PARAM_ORDER} == pin["params"]
    block = Block(pin["H"], pin["D"], pin["inter"], params).cuda()
    plan = skv.PrecisionPlan.from_codes(torch.from_numpy(a["codes"]).cuda())
    cache = skv.PackedKVCache.pack(torch.from_numpy(a["k"]).cuda(), torch.from_numpy(a["v"]).cuda(), None, 16,
                                   plan=plan)["packed_kv"]
    hidden = torch.from_numpy(a["hidden"]).cuda()
    with torch.no_grad():
        out, k_new, v_new = skv.packed_block_forward(block, hidden, cache)
        # the attention alone, on the block's own queries
        B, S, _ = hidden.shape
        q = block.q_proj(block.ln1(hidden)).view(B, S, pin["H"], pin["D"]).transpose(1, 2)
        attn = skv.packed_attention(q, cache, k_new=k_new, v_new=v_new)
    assert rel_l2(k_new.cpu().numpy(), a["k_new"]) < 1e-5
    assert rel_l2(v_new.cpu().numpy(), a["v_new"]) < 1e-5
    assert rel_l2(attn.cpu().numpy(), a["attn_out"]) < REL_L2_TOL
    assert rel_l2(out.cpu().numpy(), a["out"]) < REL_L2_TOL
