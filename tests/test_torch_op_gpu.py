"""torch.ops.fmha_b200.decode against torch's own attention
(F.scaled_dot_product_attention in fp32 on the same bf16 inputs), with GQA
expanded by repeating kv heads."""
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("b,hq,hkv,s,d", [(64, 32, 32, 16, 256), (33, 16, 16, 5, 128),
                                          (17, 32, 16, 16, 256), (8, 16, 4, 1, 128)])
def test_decode_op_vs_sdpa(cuda, b, hq, hkv, s, d):
    torch = cuda
    import torch.nn.functional as F

    import fmha_b200.torch_op  # noqa: F401
    g = torch.Generator(device="cuda").manual_seed(b * s)
    q = torch.randn(b, hq, 1, d, device="cuda", generator=g).bfloat16()
    k = torch.randn(b, hkv, s, d, device="cuda", generator=g).bfloat16()
    v = torch.randn(b, hkv, s, d, device="cuda", generator=g).bfloat16()
    o = torch.ops.fmha_b200.decode(q, k, v)
    rep = hq // hkv
    ref = F.scaled_dot_product_attention(q.float(), k.float().repeat_interleave(rep, 1),
                                         v.float().repeat_interleave(rep, 1))
    err = (o.float() - ref).abs()
    ok = (err <= 2e-3) | (err <= 1e-2 * ref.abs())
    assert o.dtype == torch.float16 and o.shape == (b, hq, 1, d)
    assert bool(ok.all()), float(err.max())
