"""tcgen05/TMEM GEMM (cdb_gemm_bf16) against a plain PyTorch fp32 reference on the GPU.

c = x @ w^T with bf16 x, w; the reference multiplies the same bf16 values in fp32. The GEMM
accumulates in fp32 and rounds once, so every element is within one bf16 rounding of the
reference plus fp32 summation-order noise: |c - ref| <= 2^-8 |ref| + 2^-12 * ||x_row|| ||w_row||.
Shapes cover the Ouro-1.4B projections (N 6144/2048/11264/2048, K 2048/5632, LM head 49152),
token counts from 1 to prefill sizes, M/N/K tails, automatic and forced K splits, and
repeated calls (split-K counters must return to zero).
"""

from __future__ import annotations

import pytest
import torch

from continuous_depth_batching_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda"


class Gemm:
    def __init__(self):
        self.ws = torch.zeros(64 << 20, dtype=torch.float32, device=DEV)
        self.ctr = torch.zeros(8192, dtype=torch.int32, device=DEV)
        self.status = torch.zeros(1, dtype=torch.int32, device=DEV)

    def __call__(self, x, w, splits=0, out=None):
        m, k = x.shape
        n = w.shape[0]
        c = torch.empty(m, n, dtype=torch.bfloat16, device=DEV) if out is None else out
        _lib.call(
            "cdb_gemm_bf16", _lib.ptr(x), x.stride(0), _lib.ptr(w), w.stride(0), _lib.ptr(c), c.stride(0), m, n, k,
            splits, _lib.ptr(self.ws), self.ws.numel(), _lib.ptr(self.ctr), self.ctr.numel(), 148,
            _lib.ptr(self.status), torch.cuda.current_stream().cuda_stream,
        )
        return c


@pytest.fixture(scope="module")
def gemm():
    return Gemm()


def _check(c, x, w):
    ref = x.float() @ w.float().t()
    bound = 2**-8 * ref.abs() + 2**-12 * (x.float().norm(dim=1)[:, None] * w.float().norm(dim=1)[None, :])
    bad = (c.float() - ref).abs() > bound
    assert not bad.any(), f"{int(bad.sum())} elements out of bound; max err {(c.float() - ref).abs().max().item():.3e}"


@pytest.mark.parametrize(
    "m,n,k",
    [
        (1, 6144, 2048), (7, 2048, 2048), (33, 11264, 2048), (64, 2048, 5632), (100, 6144, 2048),
        (256, 6144, 2048), (256, 2048, 2048), (256, 11264, 2048), (256, 2048, 5632), (96, 49152, 2048),
        (300, 768, 256), (1024, 1408, 256), (2048, 6144, 2048), (16, 256, 704), (130, 1000, 520),
    ],
)
def test_gemm_matches_fp32_reference(gemm, m, n, k):
    g = torch.Generator(device=DEV).manual_seed(m * 7 + n + k)
    x = torch.randn(m, k, device=DEV, generator=g).to(torch.bfloat16)
    w = (0.05 * torch.randn(n, k, device=DEV, generator=g)).to(torch.bfloat16)
    c = gemm(x, w)
    torch.cuda.synchronize()
    assert int(gemm.status.item()) == 0
    _check(c, x, w)


@pytest.mark.parametrize("splits", [1, 2, 5, 16])
def test_gemm_forced_splits_and_repeat(gemm, splits):
    g = torch.Generator(device=DEV).manual_seed(splits)
    x = torch.randn(200, 2048, device=DEV, generator=g).to(torch.bfloat16)
    w = (0.05 * torch.randn(2048, 2048, device=DEV, generator=g)).to(torch.bfloat16)
    first = gemm(x, w, splits=splits)
    for _ in range(3):
        again = gemm(x, w, splits=splits)
        torch.cuda.synchronize()
        assert torch.equal(first, again)  # deterministic across calls
    assert int(gemm.ctr.abs().sum().item()) == 0
    _check(first, x, w)


def test_gemm_strided_operands_and_output(gemm):
    g = torch.Generator(device=DEV).manual_seed(3)
    big = torch.randn(64, 3000, device=DEV, generator=g).to(torch.bfloat16)
    x = big[:, 8:2056]  # ld 3000, 16-byte aligned start
    w = (0.05 * torch.randn(512, 2048, device=DEV, generator=g)).to(torch.bfloat16)
    out = torch.zeros(64, 700, dtype=torch.bfloat16, device=DEV)
    gemm(x, w, out=out[:, :512])
    torch.cuda.synchronize()
    _check(out[:, :512], x, w)
    assert out[:, 512:].abs().sum().item() == 0
