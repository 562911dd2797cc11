"""MHFlashAttention / MHFlashAttentionGrad (NeuroNet.cl:16066-16277) past the golden shapes.

The golden cases pin both kernels to the reference for head dimensions up to 64.  These run every
lane-group configuration of the CUDA kernels (head dimensions up to 1000) against the oracle, a
batched full-size case against a float64 restatement of the same arithmetic, and the gradient
against the reference's formula, whose query and key gradients carry no 1/sqrt(d) factor.
"""
import numpy as np
import pytest

from oracle import kernels as K
from tests.parity import check_close
from tests.test_kernels_gpu import run_on_gpu

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("D", [96, 128, 200, 256, 520, 1000])
@pytest.mark.parametrize("mask", [0, 1])
def test_flash_head_dimensions_match_oracle(ctx, D, mask):
    Q, KV, H = 19, 23, 2
    rng = np.random.default_rng(D + 7 * mask)
    q = rng.standard_normal(Q * H * D).astype(np.float32)
    kv = rng.standard_normal(KV * 2 * H * D).astype(np.float32)
    fwd = [q, kv, np.zeros(Q * H, np.float32), np.zeros(Q * H * D, np.float32), D, KV, mask]
    got = run_on_gpu(ctx, "MHFlashAttention", fwd, (Q, D, H), (1, D, 1))
    ref = [a.copy() if isinstance(a, np.ndarray) else a for a in fwd]
    K.launch("MHFlashAttention", (Q, D, H), (1, D, 1), ref)
    check_close("out", got[3], ref[3])
    check_close("logsumexp", got[2], ref[2])
    g = (rng.standard_normal(Q * H * D) * 0.1).astype(np.float32)
    bwd = [q, np.zeros_like(q), kv, np.zeros_like(kv), ref[2], ref[3], g, D, Q, KV, mask]
    gotb = run_on_gpu(ctx, "MHFlashAttentionGrad", bwd, (max(Q, KV), D, H), (1, D, 1))
    refb = [a.copy() if isinstance(a, np.ndarray) else a for a in bwd]
    K.launch("MHFlashAttentionGrad", (max(Q, KV), D, H), (1, D, 1), refb)
    check_close("query_gr", gotb[1], refb[1])
    check_close("key_value_gr", gotb[3], refb[3])


def _attention_f64(q, kv, Q, KV, H, D, mask):
    q = q.reshape(Q, H, D).astype(np.float64)
    kv = kv.reshape(KV, 2 * H, D).astype(np.float64)
    k, v = kv[:, :H], kv[:, H:]
    s = np.einsum("qhd,khd->qkh", q, k) / np.sqrt(D)
    if mask:
        s = np.where((np.arange(Q)[:, None] <= np.arange(KV)[None, :])[:, :, None], s, -np.inf)
    m = s.max(axis=1, keepdims=True)
    p = np.exp(s - m)
    z = p.sum(axis=1, keepdims=True)
    out = np.einsum("qkh,khd->qhd", p / z, v)
    lse = (m + np.log(z))[:, 0, :]
    return out, lse, k, v


@pytest.mark.parametrize("mask", [0, 1])
def test_flash_full_size_batched(ctx, mask):
    """Two samples of 512 queries x 640 keys, 8 heads of 64: forward against float64 attention,
    then the gradient of the reference's formula against float64."""
    B, Q, KV, H, D = 2, 512, 640, 8, 64
    rng = np.random.default_rng(41 + mask)
    q = rng.standard_normal(B * Q * H * D).astype(np.float32)
    kv = rng.standard_normal(B * KV * 2 * H * D).astype(np.float32)
    fwd = [q, kv, np.zeros(B * Q * H, np.float32), np.zeros(B * Q * H * D, np.float32), D, KV, mask]
    got = run_on_gpu(ctx, "MHFlashAttention", fwd, (Q, D, H), (1, D, 1), batch=B)
    g = (rng.standard_normal(B * Q * H * D) * 0.1).astype(np.float32)
    bwd = [q, np.zeros_like(q), kv, np.zeros_like(kv), got[2], got[3], g, D, Q, KV, mask]
    gotb = run_on_gpu(ctx, "MHFlashAttentionGrad", bwd, (max(Q, KV), D, H), (1, D, 1), batch=B)
    for b in range(B):
        qs, ks = q[b * Q * H * D:(b + 1) * Q * H * D], kv[b * KV * 2 * H * D:(b + 1) * KV * 2 * H * D]
        out, lse, k, v = _attention_f64(qs, ks, Q, KV, H, D, mask)
        check_close(f"out b{b}", got[3][b * Q * H * D:(b + 1) * Q * H * D], out.reshape(-1).astype(np.float32))
        check_close(f"logsumexp b{b}", got[2][b * Q * H:(b + 1) * Q * H], lse.reshape(-1).astype(np.float32))
        # the reference's gradient: p from the saved lse, ds = p (g.v - g.o), no 1/sqrt(d) on q and k
        gq = g[b * Q * H * D:(b + 1) * Q * H * D].reshape(Q, H, D).astype(np.float64)
        o = got[3][b * Q * H * D:(b + 1) * Q * H * D].reshape(Q, H, D).astype(np.float64)
        l = got[2][b * Q * H:(b + 1) * Q * H].reshape(Q, H).astype(np.float64)
        qq = qs.reshape(Q, H, D).astype(np.float64)
        s = np.einsum("qhd,khd->qkh", qq, k) / np.sqrt(D)
        p = np.exp(np.clip(s - l[:, None, :], -120, 0))
        if mask:
            p = p * (np.arange(Q)[:, None] <= np.arange(KV)[None, :])[:, :, None]
        ds = p * (np.einsum("qhd,khd->qkh", gq, v) - (gq * o).sum(-1)[:, None, :])
        dq = np.einsum("qkh,khd->qhd", ds, k)
        dk = np.einsum("qkh,qhd->khd", ds, qq)
        dv = np.einsum("qkh,qhd->khd", p, gq)
        check_close(f"query_gr b{b}", gotb[1][b * Q * H * D:(b + 1) * Q * H * D], dq.reshape(-1).astype(np.float32))
        kvg = gotb[3][b * KV * 2 * H * D:(b + 1) * KV * 2 * H * D].reshape(KV, 2 * H, D)
        check_close(f"key_gr b{b}", kvg[:, :H], dk.astype(np.float32))
        check_close(f"value_gr b{b}", kvg[:, H:], dv.astype(np.float32))
