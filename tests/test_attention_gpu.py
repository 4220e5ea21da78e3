"""tcgen05 flash attention parity against an fp32 PyTorch softmax-attention reference.

Cases: chunk-0 self-attention (history segment empty), steady self-attention over
[history | current] (2 x 2640 keys), cross-attention over 257 context keys (one segment),
ragged segments that end mid-tile, one head and twelve heads.  Segment lengths are device
resident.  Tolerance: rel-L2 <= 1e-2, max-abs <= 2e-2 (bf16 P and output).
"""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

CASES = [
    # Lq, H, n0, n1, cap0, cap1
    (256, 2, 0, 256, 256, 256),
    (2640, 2, 2640, 2640, 2640, 2640),
    (2640, 12, 0, 2640, 2640, 2640),
    (2640, 12, 2640, 2640, 2640, 2640),
    (300, 1, 257, 0, 257, 257),
    (130, 1, 100, 37, 128, 64),
    (2640, 2, 257, 0, 257, 257),
]


def _ref(q, k, v):
    s = torch.einsum("qhd,khd->hqk", q.float(), k.float()) / math.sqrt(q.shape[-1])
    return torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), v.float()).reshape(q.shape[0], -1)


@pytest.mark.parametrize("Lq,H,n0,n1,cap0,cap1", CASES)
def test_attention(Lq, H, n0, n1, cap0, cap1):
    from fastworld_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(Lq + H + n0)
    r = lambda n: torch.randn(n, H, 128, device="cuda", generator=g).to(torch.bfloat16)
    q, k0, v0, k1, v1 = r(Lq), r(cap0), r(cap0), r(cap1), r(cap1)
    meta = torch.tensor([n0, n1], dtype=torch.int32, device="cuda")
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    out = ops.attention(q, k0, v0, k1, v1, meta, status)
    ref = _ref(q, torch.cat([k0[:n0], k1[:n1]]), torch.cat([v0[:n0], v1[:n1]]))
    torch.cuda.synchronize()
    assert int(status[0]) == 0
    err = float((out.float() - ref).norm() / ref.norm())
    assert err < 1e-2, err
    assert float((out.float() - ref).abs().max()) < 2e-2


def test_attention_deterministic():
    from fastworld_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(9)
    r = lambda n: torch.randn(n, 12, 128, device="cuda", generator=g).to(torch.bfloat16)
    q, k0, v0, k1, v1 = r(2640), r(2640), r(2640), r(2640), r(2640)
    meta = torch.tensor([2640, 2640], dtype=torch.int32, device="cuda")
    assert torch.equal(ops.attention(q, k0, v0, k1, v1, meta), ops.attention(q, k0, v0, k1, v1, meta))
