"""K1 (lema_proj_codes): tcgen05 projection GEMM with the sign-pack epilogue.

The reference computes z = x @ w.T with a bf16 cuBLAS GEMM and packs sign bits
(code/lema/model.py:168-175, 224-227; code/lema/attention.py:82-97); no reference test pins
z. Codes are checked against an fp64 z of the same bf16 inputs under the tolerance rule for
codes: a bit may differ from the exact sign only where |z_d| < 1e-3 * ||z_row||_2 (z_row =
that head's 32 pre-activations). The same rule is applied to the reference's own recipe
(torch bf16 GEMM + pack_codes), and flips are counted and reported.
"""
import pytest
import torch

from latest_exact_match_attention_b200 import pack_codes, proj_codes

pytestmark = pytest.mark.gpu

TOL = 1e-3


def bits_of(codes: torch.Tensor) -> torch.Tensor:
    c = codes.to(torch.int64) & 0xFFFFFFFF
    return ((c[..., None] >> torch.arange(32, device=c.device)) & 1).bool()


def exact_z(x, w, hq, hk):
    """fp64 pre-activations [B, heads, T, 32] of the bf16 inputs."""
    B, T, _ = x.shape
    z = (x.double() @ w.double().T).view(B, T, hq + hk, 32).permute(0, 2, 1, 3)
    return z[:, :hq], z[:, hq:]


def flips(codes, z):
    """Number of sign bits that differ from the exact z; fails on any flip outside the band."""
    exact = z >= 0
    got = bits_of(codes)
    diff = got != exact
    band = z.abs() < TOL * z.norm(dim=-1, keepdim=True)
    bad = diff & ~band
    assert not bool(bad.any()), f"{int(bad.sum())} flipped bits outside |z| < {TOL}*||z||"
    return int(diff.sum())


def make(B, T, dim, hq, hk, dev, seed=0, zero_rows=0):
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn((B, T, dim), generator=g, device=dev).to(torch.bfloat16)
    w = (0.02 * torch.randn(((hq + hk) * 32, dim), generator=g, device=dev)).to(torch.bfloat16)
    if zero_rows:
        x[:, :zero_rows] = 0
    return x, w


CASES = [
    # B, T, dim, hq, hk: tails in rows (M % 128) and columns (heads % 8), GQA, many tiles
    (2, 200, 128, 3, 2),
    (1, 64, 64, 1, 1),
    (4, 1024, 1024, 8, 8),
    (2, 1000, 512, 4, 2),
    (2, 2048, 1024, 64, 64),
    (5, 2048, 256, 4, 4),      # picks the 128-column tile (64 and 256 are picked above)
    (256, 1, 1536, 64, 64),    # a decode step: 256 rows, the 64-column tile
]


@pytest.mark.parametrize("B,T,dim,hq,hk", CASES)
def test_proj_codes_vs_exact_sign(cuda, B, T, dim, hq, hk):
    x, w = make(B, T, dim, hq, hk, cuda, seed=B * 7 + hq)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    qc, kc = proj_codes(x, w, hq, hk, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert qc.shape == (B, hq, T) and kc.shape == (B, hk, T)
    zq, zk = exact_z(x, w, hq, hk)
    n_bits = (zq.numel() + zk.numel())
    f = flips(qc, zq) + flips(kc, zk)
    assert f <= max(8, n_bits // 100000), f"{f} flips in {n_bits} bits"
    # the reference's recipe (bf16 GEMM, then pack) is held to the same rule
    zb = (x @ w.T).view(B, T, hq + hk, 32).permute(0, 2, 1, 3)
    rq, rk = pack_codes(zb[:, :hq], narrow=True), pack_codes(zb[:, hq:], narrow=True)
    flips(rq, zq)
    flips(rk, zk)


def test_proj_codes_zero_rows_and_repeat(cuda):
    # all-zero rows give z = 0 exactly: every bit set (0 >= 0), as pack_codes does
    x, w = make(2, 384, 256, 5, 3, cuda, seed=3, zero_rows=130)
    qc, kc = proj_codes(x, w, 5, 3)
    qc2, kc2 = proj_codes(x, w, 5, 3)
    torch.cuda.synchronize()
    assert torch.equal(qc, qc2) and torch.equal(kc, kc2)
    assert bool((qc[:, :, :130] == -1).all()) and bool((kc[:, :, :130] == -1).all())
    zq, zk = exact_z(x, w, 5, 3)
    flips(qc, zq)
    flips(kc, zk)


@pytest.mark.parametrize("B,T,dim,H,dv", [(2, 300, 256, 8, 32), (256, 1, 1536, 64, 24), (4, 1024, 1024, 16, 64)])
def test_value_columns_in_one_gemm(cuda, B, T, dim, H, dv):
    """lema_proj_codes_v: the q/k codes and the value projection of the same (normalised)
    rows in one tcgen05 GEMM. The codes obey the flip rule against an fp64 z with no flip
    outside the band (the same rows and weights as the codes-only kernel, so the same
    accumulation); the value columns equal the fp64 product to bf16 rounding, times the row
    scale when one is given."""
    from latest_exact_match_attention_b200.attention import proj_codes_v
    g = torch.Generator(device=cuda).manual_seed(B + H)
    x = torch.randn((B, T, dim), generator=g, device=cuda).to(torch.bfloat16)
    w = (0.05 * torch.randn(((2 * H) * 32 + H * dv, dim), generator=g, device=cuda)).to(torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    qc, kc, v = proj_codes_v(x, w, H, H, H * dv, status=status)
    rs = (0.5 + torch.rand(B * T, generator=g, device=cuda)).float()
    _, _, v2 = proj_codes_v(x, w, H, H, H * dv, row_scale=rs, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    zq, zk = exact_z(x, w[: 2 * H * 32], H, H)
    print(f"flips (all inside the band): {flips(qc, zq) + flips(kc, zk)} of {zq.numel() + zk.numel()} bits")
    q1, k1 = proj_codes(x, w[: 2 * H * 32], H, H)
    assert torch.equal(q1, qc) and torch.equal(k1, kc)
    zv = (x.double() @ w[2 * H * 32:].double().T).float()
    torch.testing.assert_close(v.float(), zv, rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(v2.float(), zv * rs.view(B, T, 1), rtol=1e-2, atol=1e-2)
