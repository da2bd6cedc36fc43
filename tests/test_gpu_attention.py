"""GPU: the short-key attention kernel (``qi_b200_attention_short``) against an
fp64 softmax(Q K^T / sqrt(d)) V of the same bf16 inputs.

The kernel rounds the probabilities to bf16 before the P V product, as flash
attention kernels do; tolerance: relative Frobenius error <= 1e-2 and max
abs error <= 3e-2 (unit-variance V).  Shapes: the DiT step's cross-attention
(3120 video or 32 action queries x 128 context keys, 24 heads), plus ragged
query / key counts, one key, large logits, strided rows; more than 128 keys
is refused.
"""

import pytest
import torch

from qi_b200 import _lib, kernels as K

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module", autouse=True)
def _device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    _lib.load()
    torch.cuda.set_device(0)
    yield
    torch.cuda.synchronize()
    st = _lib.device_status(clear=True)
    assert st[0] == 0, f"device status word reports a timed-out wait: {st}"


def _ref(q, k, v, heads):
    sq, sk = q.shape[0], k.shape[0]
    qh = q.double().view(sq, heads, 128).transpose(0, 1)
    kh = k.double().view(sk, heads, 128).transpose(0, 1)
    vh = v.double().view(sk, heads, 128).transpose(0, 1)
    p = torch.softmax(torch.bmm(qh, kh.transpose(1, 2)) * 128 ** -0.5, -1)
    return torch.bmm(p, vh).transpose(0, 1).reshape(sq, heads * 128)


@pytest.mark.parametrize("sq,sk,heads,qmul", [
    (3120, 128, 24, 1.0),   # DiT cross-attention, video queries
    (32, 128, 24, 1.0),     # action queries
    (1, 1, 2, 1.0),
    (129, 65, 1, 1.0),
    (300, 120, 3, 1.0),
    (257, 100, 4, 6.0),     # large logits: the row max matters
    (1000, 128, 40, 1.0),   # items not a multiple of the grid; several heads per CTA
])
def test_attention_short_matches_fp64(sq, sk, heads, qmul):
    g = torch.Generator(device="cpu").manual_seed(sq * 7 + sk)
    w = heads * 128
    q = (torch.randn(sq, w, generator=g) * qmul).to(torch.bfloat16).to(DEV)
    k = torch.randn(sk, w, generator=g).to(torch.bfloat16).to(DEV)
    v = torch.randn(sk, w, generator=g).to(torch.bfloat16).to(DEV)
    o = K.attention_short(q, k, v.t().contiguous(), heads)
    torch.cuda.synchronize()
    want = _ref(q, k, v, heads)
    d = o.double() - want
    rel = (d.norm() / want.norm()).item()
    assert rel <= 1e-2, rel
    assert d.abs().max().item() <= 3e-2, d.abs().max().item()
    # deterministic: the same bits on a second launch
    assert torch.equal(o, K.attention_short(q, k, v.t().contiguous(), heads))


def test_attention_short_strided_rows_and_out():
    """q and k as column slices of wider row blocks (a fused QKV output), the
    result written into a slice of a larger tensor."""
    heads, sq, sk = 8, 500, 128
    w = heads * 128
    g = torch.Generator(device="cpu").manual_seed(5)
    qkv = torch.randn(sq, 3 * w, generator=g).to(torch.bfloat16).to(DEV)
    kv = torch.randn(sk, 2 * w, generator=g).to(torch.bfloat16).to(DEV)
    q, k, v = qkv[:, :w], kv[:, :w], kv[:, w:]
    big = torch.zeros(sq + 10, w, dtype=torch.bfloat16, device=DEV)
    K.attention_short(q, k, v.t().contiguous(), heads, out=big[5:5 + sq])
    torch.cuda.synchronize()
    assert torch.equal(big[5:5 + sq], K.attention_short(q.contiguous(), k.contiguous(), v.t().contiguous(), heads))
    assert big[:5].abs().sum().item() == 0 and big[5 + sq:].abs().sum().item() == 0
    d = big[5:5 + sq].double() - _ref(q, k, v, heads)
    assert d.abs().max().item() <= 3e-2


def test_attention_short_matches_torch_sdpa():
    """Same inputs through torch's scaled_dot_product_attention (bf16): the two
    bf16 results agree to the tolerance above."""
    heads, sq, sk = 24, 3120, 128
    w = heads * 128
    g = torch.Generator(device="cpu").manual_seed(9)
    q = torch.randn(sq, w, generator=g).to(torch.bfloat16).to(DEV)
    k = torch.randn(sk, w, generator=g).to(torch.bfloat16).to(DEV)
    v = torch.randn(sk, w, generator=g).to(torch.bfloat16).to(DEV)
    o = K.attention_short(q, k, v.t().contiguous(), heads)
    t = torch.nn.functional.scaled_dot_product_attention(
        q.view(1, sq, heads, 128).transpose(1, 2), k.view(1, sk, heads, 128).transpose(1, 2),
        v.view(1, sk, heads, 128).transpose(1, 2)).transpose(1, 2).reshape(sq, w)
    d = (o.float() - t.float())
    assert (d.norm() / t.float().norm()).item() <= 1e-2
    assert d.abs().max().item() <= 3e-2


def test_attention_short_rejects_bad_shapes():
    q = torch.zeros(16, 256, dtype=torch.bfloat16, device=DEV)
    k = torch.zeros(300, 256, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(Exception):
        K.attention_short(q, k[:129], torch.zeros(256, 136, dtype=torch.bfloat16, device=DEV)[:, :129], 2)  # > 128 keys
    with pytest.raises(ValueError):
        K.attention_short(q, k[:8], torch.zeros(256, 9, dtype=torch.bfloat16, device=DEV), 2)  # vt shape
