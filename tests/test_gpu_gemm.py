"""tcgen05 GEMMs through the C ABI against fp32 / exact-integer references."""

import pytest
import torch

from oracle import compare_outputs, int_gemm_ref, quant_rows_ref, quant_weight_ref
from tiktok_techjam_2026_track3_b200 import ops

pytestmark = pytest.mark.gpu

DT = {"fp16": torch.float16, "bf16": torch.bfloat16}


@pytest.fixture(autouse=True)
def _no_tf32():
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = old


def _rand(shape, g, scale, dtype):
    return (torch.randn(*shape, generator=g) * scale).to(dtype).cuda()


SHAPES = [(128, 256, 64), (200, 96, 72), (1, 32, 8), (1000, 768, 256), (777, 512, 1000),
          (4096, 3072, 1024), (2048, 1024, 4096),
          # more 256 x 256 tiles than CTA pairs, the last partial wave small enough to run as
          # 256 x 128 column halves (80 tiles on 74 pairs: 6 tiles -> 12 halves), ragged rows
          (10163, 512, 320)]


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("m,n,k", SHAPES)
def test_linear_bias(dt, m, n, k):
    g = torch.Generator().manual_seed(m * 31 + n * 7 + k)
    x, w = _rand((m, k), g, 1.0, DT[dt]), _rand((n, k), g, k ** -0.5, DT[dt])
    b = _rand((n,), g, 0.1, DT[dt])
    y = ops.linear(x, w, b)
    ref = x.float() @ w.float().T + b.float()
    rep = compare_outputs(ref, y.float())
    assert rep.passed, str(rep)
    ops.check_device_status(x.device)


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("m,n,k", [(300, 256, 128), (2048, 1024, 1024),
                                   # more tiles than CTA pairs (or CTAs), last row block ragged:
                                   # an epilogue warp requests its next tile's first residual box
                                   # before that tile's accumulator is ready
                                   (16461, 1024, 256), (16400, 256, 128), (64, 40960, 64),
                                   # tail tiles as column halves (see SHAPES)
                                   (10163, 512, 320), (16384, 1024, 1024)])
def test_linear_residual_rowmask(dt, m, n, k):
    g = torch.Generator().manual_seed(11)
    x, w = _rand((m, k), g, 1.0, DT[dt]), _rand((n, k), g, k ** -0.5, DT[dt])
    b, res = _rand((n,), g, 0.1, DT[dt]), _rand((m, n), g, 1.0, DT[dt])
    mask = torch.rand(m, generator=g) > 0.3
    y = ops.linear(x, w, b, residual=res, row_mask=mask.cuda())
    attn = (x.float() @ w.float().T + b.float()).masked_fill(~mask.cuda()[:, None], 0)
    rep = compare_outputs(res.float() + attn, y.float())
    assert rep.passed, str(rep)
    # masked rows are exactly the residual
    assert torch.equal(y[~mask.cuda()], res[~mask.cuda()])
    # no residual: masked rows are exactly zero
    y0 = ops.linear(x, w, b, row_mask=mask.cuda())
    assert torch.count_nonzero(y0[~mask.cuda()]) == 0


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
def test_quant_rows_bit_exact(dt):
    g = torch.Generator().manual_seed(3)
    x = torch.randn(1031, 1024, generator=g)
    x[5] = 0           # clamp path
    x[9] *= 1e-7       # tiny rows
    x[17, 3] = 300.0   # outlier
    xd = x.to(DT[dt]).cuda()
    q, s = ops.int8_quant_rows(xd)
    q_ref, s_ref = quant_rows_ref(xd.float().cpu())
    assert torch.equal(s.cpu(), s_ref)
    assert torch.equal(q.cpu(), q_ref)


@pytest.mark.parametrize("m,n,k", [(128, 256, 128), (300, 96, 160), (1, 32, 16), (2048, 1536, 4096),
                                   (4096, 4096, 4096), (10163, 512, 320)])
def test_int8_gemm_s32_bit_exact(m, n, k):
    g = torch.Generator().manual_seed(m + n + k)
    a = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8).cuda()
    w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8).cuda()
    acc = ops.int8_gemm_s32(a, w)
    assert torch.equal(acc, int_gemm_ref(a, w))
    ops.check_device_status(a.device)


@pytest.mark.parametrize("out", ["bf16", "fp16"])
@pytest.mark.parametrize("m,n,k", [(513, 768, 256), (4096, 3072, 1024), (10163, 512, 320)])
def test_int8_linear_dequant(out, m, n, k):
    """Dequant epilogue follows the recipe's op order, so it is bit-exact in
    fp32 and therefore after rounding to the output dtype."""
    g = torch.Generator().manual_seed(5)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).cuda()
    wf = torch.randn(n, k, generator=g) * 0.02
    w8, s_w = quant_weight_ref(wf)
    w8, s_w = w8.cuda(), s_w.cuda()
    bias = (torch.randn(n, generator=g) * 0.02).cuda()
    a8, s_a = ops.int8_quant_rows(x)
    y = ops.int8_linear(a8, s_a, w8, s_w, bias, DT[out])
    ref = int_gemm_ref(a8, w8).float() * (s_a[:, None] * s_w[None, :]) + bias[None, :]
    assert torch.equal(y, ref.to(DT[out]))
    res = torch.randn(m, n, generator=g).to(DT[out]).cuda()
    mask = (torch.rand(m, generator=g) > 0.2).cuda()
    y2 = ops.int8_linear(a8, s_a, w8, s_w, bias, DT[out], residual=res, row_mask=mask)
    ref2 = res.float() + ref.masked_fill(~mask[:, None], 0)
    assert torch.equal(y2, ref2.to(DT[out]))


def test_weight_quantizer_matches_recipe():
    g = torch.Generator().manual_seed(9)
    w = torch.randn(96, 256, generator=g) * 0.02
    w[4] = 0
    q, s = ops.quantize_weight(w.cuda())
    q_ref, s_ref = quant_weight_ref(w)
    assert torch.equal(q.cpu(), q_ref) and torch.equal(s.cpu(), s_ref)


@pytest.mark.parametrize("dt", ["fp16", "bf16"])
@pytest.mark.parametrize("m,n,k,kc", [(512, 1024, 1024, 128), (777, 512, 512, 64), (4096, 4096, 4096, 512)])
def test_linear_kchunked_matches_plain(dt, m, n, k, kc):
    """Input stored K-chunk-major [k/kc, m, kc] (the head-sharded gather layout)."""
    g = torch.Generator().manual_seed(m + kc)
    x, w = _rand((m, k), g, 1.0, DT[dt]), _rand((n, k), g, k ** -0.5, DT[dt])
    b, res = _rand((n,), g, 0.1, DT[dt]), _rand((m, n), g, 1.0, DT[dt])
    chunks = x.view(m, k // kc, kc).permute(1, 0, 2).contiguous()
    y = ops.linear_kchunked(chunks, w, b, residual=res)
    y_plain = ops.linear(x, w, b, residual=res)
    assert torch.equal(y, y_plain)  # same tiles, same order of accumulation
    rep = compare_outputs(res.float() + x.float() @ w.float().T + b.float(), y.float())
    assert rep.passed, str(rep)
