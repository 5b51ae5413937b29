"""The transformer block on the sm_100a kernels (BaselineTransformerBlock,
torch_transformer_benchmark.py:125-145): LayerNorm, GEMM with exact-GELU
epilogue, and the whole block through ttj_transformer_block_fwd, against fp32
restatements on the same rounded inputs and against the reference module's
own 16-bit run.
"""

import pytest
import torch
import torch.nn.functional as F

from oracle import compare_outputs
from oracle.block_ref import BaselineTransformerBlockRef
from tiktok_techjam_2026_track3_b200 import ops, plugin

pytestmark = pytest.mark.gpu

DT = {"fp16": torch.float16, "bf16": torch.bfloat16}
# one rounding of a value of magnitude ~1 in the output dtype, twice
TOL = {"fp16": 2 * 2.0 ** -11, "bf16": 2 * 2.0 ** -8}


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("rows,d", [(1, 64), (37, 192), (1031, 1024), (64, 4096), (5, 8192)])
def test_layernorm_matches_fp32(dt, rows, d):
    dtype = DT[dt]
    g = torch.Generator().manual_seed(rows * 7 + d)
    x = (torch.randn(rows, d, generator=g) * 3 + 2).to(dtype)   # non-zero mean: centring matters
    w = (1 + 0.1 * torch.randn(d, generator=g)).to(dtype)
    b = (0.1 * torch.randn(d, generator=g)).to(dtype)
    mask = torch.rand(rows, generator=g) > 0.2
    mask[0] = True
    eps = 1e-5
    out = ops.layernorm(x.cuda(), w.cuda(), b.cuda(), eps, row_mask=mask.cuda()).float().cpu()
    ref = F.layer_norm(x.float(), (d,), w.float(), b.float(), eps)
    keep = mask[:, None].expand_as(ref)
    err = (out - ref).abs()[keep]
    bound = TOL[dt] * ref.abs()[keep].clamp_min(1.0)
    assert bool((err <= bound).all()), f"max err {err.max():.3g}"
    assert bool((out[~mask] == 0).all())
    # no mask: every row normalised
    out2 = ops.layernorm(x.cuda(), w.cuda(), b.cuda(), eps).float().cpu()
    assert bool(((out2 - ref).abs() <= TOL[dt] * ref.abs().clamp_min(1.0)).all())


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("m,n,k", [(300, 512, 256), (4096, 2048, 1024), (64, 96, 64)])
def test_linear_gelu_matches_fp32(dt, m, n, k):
    dtype = DT[dt]
    g = torch.Generator().manual_seed(m + n + k)
    x = torch.randn(m, k, generator=g).to(dtype)
    w = (torch.randn(n, k, generator=g) * k ** -0.5).to(dtype)
    b = (0.1 * torch.randn(n, generator=g)).to(dtype)
    out = ops.linear_gelu(x.cuda(), w.cuda(), b.cuda()).float().cpu()
    ref = F.gelu(x.float() @ w.float().T + b.float(), approximate="none")
    rep = compare_outputs(ref, out)
    assert rep.passed, str(rep)


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
def test_gelu_epilogue_matches_exact_erf(dt):
    """The GELU epilogue against exact GELU evaluated in float64 (through erfc,
    so the negative tail is exact) on the same pre-activations: a one-hot x
    makes every accumulator exactly one weight.  The epilogue's erfc (fractional
    error < 1.2e-7) must give the correctly rounded 16-bit value almost
    everywhere and be off by at most one unit in the last place anywhere --
    closer than torch's own fp32 GELU, which loses the tail to cancellation in
    1 + erf(z), as the last assertion records."""
    dtype = DT[dt]
    K, N, M = 64, 1024, 256
    vals = torch.linspace(-12.0, 12.0, K * N).to(dtype)          # pre-activations, exact in dtype
    w = vals.view(N, K)
    x = torch.zeros(M, K, dtype=dtype)
    x[torch.arange(M), torch.arange(M) % K] = 1.0                 # row m picks column m % K of w
    b = torch.zeros(N, dtype=dtype)
    out = ops.linear_gelu(x.cuda(), w.cuda(), b.cuda()).cpu().double()
    pre = w.double().T[torch.arange(M) % K]                       # [M, N] exact pre-activations
    exact = (0.5 * pre * torch.special.erfc(-pre / 2.0 ** 0.5)).to(dtype).double()
    ulp = (exact.abs() * 2.0 ** (-10 if dt == "fp16" else -7)).clamp_min(2.0 ** -24)
    diff = (out - exact).abs()
    assert bool((diff <= ulp).all()), f"max diff {diff.max():.3g}"
    assert float((diff == 0).double().mean()) > 0.99
    torch_fp32 = F.gelu(pre.float(), approximate="none").to(dtype).double()
    assert float((torch_fp32 - exact).abs().max()) <= 2e-3          # same tolerance as the layer


def _block(D, H, Fdim, seed):
    torch.manual_seed(seed)
    blk = BaselineTransformerBlockRef(D, H, Fdim)
    with torch.no_grad():
        for p in blk.parameters():
            p.normal_(0.0, 0.02)
        blk.norm1.weight.add_(1.0)
        blk.norm2.weight.add_(1.0)
    return blk


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("D,H,Fdim,masked", [(256, 4, 1024, False), (256, 4, 1024, True),
                                             (512, 4, 2048, True), (1024, 16, 4096, False)])
def test_block_against_fp32_and_reference_run(dt, D, H, Fdim, masked):
    dtype = DT[dt]
    B, S = 2, 320
    blk = _block(D, H, Fdim, 1234 + D)
    x = torch.randn(B, S, D, generator=torch.Generator().manual_seed(D)).to(dtype)
    mask = None
    if masked:
        mask = torch.ones(B, S, dtype=torch.bool)
        mask[1, 250:] = False
    # fp32 target on the same rounded parameters and input
    ref32 = BaselineTransformerBlockRef(D, H, Fdim)
    ref32.load_state_dict({k: v.to(dtype).float() for k, v in blk.state_dict().items()})
    with torch.inference_mode():
        target = ref32(x.float(), mask, True)
    # the reference module's own 16-bit run (the benchmark's baseline side)
    ref16 = BaselineTransformerBlockRef(D, H, Fdim)
    ref16.load_state_dict(blk.state_dict())
    ref16 = ref16.to(device="cuda", dtype=dtype).eval()
    # ours
    blk16 = BaselineTransformerBlockRef(D, H, Fdim)
    blk16.load_state_dict(blk.state_dict())
    blk16 = blk16.to(device="cuda", dtype=dtype).eval()
    mcuda = None if mask is None else mask.cuda()
    with torch.inference_mode():
        base = ref16(x.cuda(), mcuda, True, in_dtype=True).float().cpu()
        out = plugin.block_forward(blk16, x.cuda(), mcuda, True).float().cpu()
    if mask is not None:
        assert bool((out[~mask] == 0).all())
    err_ours = (out - target).abs()
    err_base = (base - target).abs()
    print(f"{dt} D{D} F{Fdim}: ours max {err_ours.max():.3g} mean {err_ours.mean():.3g}; "
          f"reference {dt} run max {err_base.max():.3g} mean {err_base.mean():.3g}")
    assert float(err_ours.mean()) <= 1.5 * float(err_base.mean()) + 1e-4
    assert float(err_ours.max()) <= 2.0 * float(err_base.max()) + 1e-3


@pytest.mark.parametrize("rows,d", [(1, 32), (37, 128), (1031, 1024), (64, 4096)])
def test_layernorm_fp32_stream(rows, d):
    """LayerNorm over fp32 rows (the residual stream of an fp32 model) with fp32
    gamma/beta, written in fp32: against torch's fp32 LayerNorm."""
    g = torch.Generator().manual_seed(rows + d)
    x = torch.randn(rows, d, generator=g) * 3 + 2
    w = 1 + 0.1 * torch.randn(d, generator=g)
    b = 0.1 * torch.randn(d, generator=g)
    mask = torch.rand(rows, generator=g) > 0.2
    mask[0] = True
    out = ops.layernorm(x.cuda(), w.cuda(), b.cuda(), 1e-5, row_mask=mask.cuda()).cpu()
    ref = F.layer_norm(x, (d,), w, b, 1e-5)
    assert out.dtype == torch.float32
    torch.testing.assert_close(out[mask], ref[mask], rtol=2e-5, atol=2e-5)
    assert bool((out[~mask] == 0).all())


@pytest.mark.parametrize("masked", [False, True])
def test_block_fp32_stream_against_fp32_module(masked):
    """One block of an fp32 model (fp32 residual stream, fp16 tensor-core
    operands) against the fp32 reference block on the unrounded parameters."""
    B, S, D, H, Fdim = 2, 384, 256, 4, 1024
    torch.manual_seed(3)
    blk = BaselineTransformerBlockRef(D, H, Fdim).eval()
    x = torch.randn(B, S, D, generator=torch.Generator().manual_seed(D))
    mask = None
    if masked:
        mask = torch.ones(B, S, dtype=torch.bool)
        mask[1, 250:] = False
    with torch.inference_mode():
        ref = blk(x, mask, True)
    dev = blk.to("cuda")
    with torch.inference_mode():
        out = plugin.block_forward(dev, x.cuda(), None if mask is None else mask.cuda(), True)
    assert out.dtype == torch.float32
    rep = compare_outputs(ref, out.cpu())
    assert rep.passed, str(rep)
