"""Expert math pinned to the reference's compute library: vLLM's
``fused_experts`` (the call of the reference's paged forward,
src/wisp/integrations/vllm/fused_moe.py:1106-1118) run on a GPU for seeded
cases by ``tests/golden/make_vllm_golden.py``; the inputs are rebuilt here
from the seeds and checked against the stored checksums.

* CPU: the fp32 oracle (vLLM's bf16 storage points) against vLLM's outputs,
  max-abs <= 1e-2 and mean-rel <= 1e-3, the tolerance of every parity test.
* GPU: this library's layer, resident and paged, on the CUDA-core and the
  tensor-core kernels, against vLLM's outputs with the same tolerance."""
import os

import numpy as np
import pytest
import torch

from oracle.moe import compare, moe_reference
from tests.golden.make_vllm_golden import CASES, case_tensors, checksum

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "vllm_fused_experts.npz")
MAX_ABS, MEAN_REL = 1e-2, 1e-3


def _case(case):
    name, E, H, I, T, K, cap, seed = case
    d = np.load(GOLD)
    tensors = case_tensors(E, H, I, T, K, cap, seed)
    np.testing.assert_array_equal(checksum(*tensors), d[name + "/checksum"],
                                  err_msg="seeded inputs differ from the ones vLLM saw")
    out = torch.from_numpy(d[name + "/out"]).view(torch.bfloat16)
    return tensors, out


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_oracle_matches_vllm_fused_experts(case):
    (w13, w2, x, w, ids, _), vllm_out = _case(case)
    c = compare(vllm_out, moe_reference(x, w13, w2, w, ids))
    assert c["max_abs"] <= MAX_ABS and c["mean_rel"] <= MEAN_REL, c


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
@pytest.mark.parametrize("cls", ["cuda", "tc"])
def test_layer_matches_vllm_fused_experts(case, cls):
    from wisp_b200.integrations.vllm.fused_moe import WispMoEState
    name, E, H, I, T, K, cap, seed = case
    (w13, w2, x, w, ids, _), vllm_out = _case(case)
    dev = torch.device("cuda:0")
    for mode, c_exp in (("resident", E), ("paged", cap)):
        st = WispMoEState(w13, w2, c_exp, mode, dev, 0)
        if mode == "resident":
            st.prime_identity()
        st.configure(compute_class=cls)
        out = st.forward(x.to(dev), w.to(dev), ids.to(dev))
        st.synchronize()
        c = compare(out.cpu(), vllm_out.float())
        assert c["max_abs"] <= MAX_ABS and c["mean_rel"] <= MEAN_REL, (mode, c)
        st.close()
