"""The router kernel (``wisp_route_topk`` / ``select_experts``) against torch's
softmax + topk + renormalise on the same GPU (the routing of the reference's
paged forward, vLLM select_experts at fused_moe.py:1054-1076).

Ids: the k largest of torch's fp32 softmax probabilities in descending order,
ties to the lower expert id -- identical to torch.topk on every row without
tied probabilities (torch.topk's order among equal values is not defined: on
a B200 it returns tie runs ascending, descending and mixed).  The selected
probabilities within 1 ulp of torch's fp32 softmax; renormalised weights
within 1 ulp of the exact renormalisation of torch's probabilities (computed
in float64); the forward from logits byte-identical to the forward from the
routed weights and ids."""
import pytest
import torch

from wisp_b200 import workloads as wl

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def torch_route(logits, k, renorm=True):
    p = torch.softmax(logits.float(), dim=-1)
    w, ids = torch.topk(p, k, dim=-1)
    if renorm:
        w = w / w.sum(dim=-1, keepdim=True)
    return w, ids.to(torch.int32)


def expected_ids(p, k):
    """Top-k of each row of p by (probability descending, id ascending)."""
    E = p.shape[1]
    return torch.tensor([sorted(range(E), key=lambda e: (-row[e], e))[:k] for row in p.cpu().tolist()],
                        dtype=torch.int32)


def untied_rows(p, k):
    """Rows whose k + 1 largest probabilities are all different."""
    v, _ = torch.topk(p.cpu(), min(k + 1, p.shape[1]), dim=-1)
    return [bool((v[r][1:] != v[r][:-1]).all()) for r in range(v.shape[0])]


def ulps(a, b):
    """Distance in units in the last place of b (fp32)."""
    ia = a.contiguous().view(torch.int32).long()
    ib = b.contiguous().view(torch.int32).long()
    return (ia - ib).abs()


@pytest.mark.parametrize("T,E,k,renorm,dtype", [
    (256, 128, 8, True, torch.float32),     # config 1 (Qwen3-30B-A3B)
    (512, 128, 8, True, torch.bfloat16),
    (64, 8, 2, True, torch.float32),        # Mixtral-8x7B
    (33, 1024, 16, False, torch.float32),
    (7, 60, 4, True, torch.float32),
])
def test_route_matches_torch(T, E, k, renorm, dtype):
    from wisp_b200.integrations.vllm.fused_moe import select_experts
    logits = (wl.router_logits(T, E, seed=T + E) * 2).to(dtype).to(DEV)
    w, ids = select_experts(logits, k, renorm)
    p, tids = torch_route(logits, k, renorm=False)
    full = torch.softmax(logits.float(), dim=-1)
    torch.cuda.synchronize()
    assert torch.equal(ids.cpu(), expected_ids(full, k))
    for r, clean in enumerate(untied_rows(full, k)):
        if clean:
            assert torch.equal(ids[r], tids[r]), r
    if renorm:
        exact = (p.double() / p.double().sum(-1, keepdim=True)).float()
        assert int(ulps(w, exact).max()) <= 1, float((w - exact).abs().max())
        pw, _ = select_experts(logits, k, False)
        assert int(ulps(pw, p).max()) <= 1
    else:
        assert int(ulps(w, p).max()) <= 1, float((w - p).abs().max())


def test_route_ties_take_the_lower_id():
    from wisp_b200.integrations.vllm.fused_moe import select_experts
    T, E, k = 16, 64, 8
    g = torch.Generator().manual_seed(5)
    logits = torch.randint(-3, 3, (T, E), generator=g).float()   # many equal logits per row
    w, ids = select_experts(logits.to(DEV), k)
    p = torch.softmax(logits, dim=-1)
    for t in range(T):
        order = sorted(range(E), key=lambda e: (-float(p[t, e]), e))[:k]
        assert ids[t].tolist() == order, t
    assert torch.equal(ids.cpu(), expected_ids(torch.softmax(logits.to(DEV), -1), k))


def test_forward_from_logits_matches_routed_forward():
    from wisp_b200.integrations.vllm.fused_moe import WispMoEState, select_experts
    E, H, I, K, T = 32, 512, 256, 8, 12
    g = torch.Generator().manual_seed(3)
    w13 = (torch.randn(E, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(E, H, I, generator=g) * 0.02).to(torch.bfloat16)
    st = WispMoEState(w13, w2, 16, "paged", DEV, 0)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
    logits = wl.router_logits(T, E, seed=9).to(DEV)
    a = st.forward_logits(x, logits, K)
    w, ids = select_experts(logits, K)
    b = st.forward(x, w, ids)
    st.synchronize()
    assert torch.equal(a, b)
    st.close()


def test_route_rejects_bad_shapes():
    from wisp_b200 import _lib
    L = _lib.lib()
    assert L.wisp_route_topk(None, 0, 4, 2048, 8, 1, None, None, None) == _lib.WISP_ERR_INVALID
    assert L.wisp_route_topk(None, 0, 4, 8, 9, 1, None, None, None) == _lib.WISP_ERR_INVALID
