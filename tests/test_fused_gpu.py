"""Fused residual-add + RMSNorm and SwiGLU activation vs the oracle."""
import numpy as np
import pytest
import torch

from oracle import kv_store as okv
from oracle.bf16 import bf16

pytestmark = pytest.mark.gpu


def _t(x):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(torch.bfloat16).cuda()


@pytest.mark.parametrize("T,H", [(1, 1024), (37, 4096), (512, 5120)])
def test_add_rmsnorm_bit_exact(T, H):
    from vllm_b200.kernels.fused import add_rmsnorm
    rng = np.random.default_rng(T + H)
    x = bf16(rng.standard_normal((T, H)) * 3)
    res = bf16(rng.standard_normal((T, H)))
    w = bf16(1 + 0.1 * rng.standard_normal(H))
    r_ref = bf16(x + res)                         # attn_output += x in bf16
    y_ref = okv.rmsnorm(r_ref, w, 1e-6)
    r, y = add_rmsnorm(_t(x), _t(w), 1e-6, residual=_t(res))
    y2 = add_rmsnorm(_t(x), _t(w), 1e-6)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(r.float().cpu().numpy(), r_ref)
    np.testing.assert_array_equal(y.float().cpu().numpy(), y_ref)
    np.testing.assert_array_equal(y2.float().cpu().numpy(), okv.rmsnorm(x, w, 1e-6))


def test_silu_mul_matches_two_roundings():
    from vllm_b200.kernels.fused import silu_mul
    rng = np.random.default_rng(1)
    T, I = 33, 3072
    gu = bf16(rng.standard_normal((T, 2 * I)) * 4)
    g, u = gu[:, :I], gu[:, I:]
    ref = bf16(bf16(g / (1 + np.exp(-g.astype(np.float64)))) * u)
    out = silu_mul(_t(gu)).float().cpu().numpy()
    diff = out != ref
    # expf vs exp may differ in the last fp32 bit: at most 1 bf16 ulp on rare elements
    assert diff.mean() < 1e-3
    np.testing.assert_allclose(out, ref, rtol=2 ** -7, atol=1e-6)
