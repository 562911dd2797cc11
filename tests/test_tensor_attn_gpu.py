"""Parity of the tensor-core multi-head attention kernels (tcgen05, 3xTF32) behind MHAttentionScore,
MHAttentionOut and MHAttentionInsideGradients.

They take a head dimension of 32, at most 128 units and units a multiple of 4: the shapes below
cover a full 128-unit tile, the 120-unit encoder tile (rows 120..127 of a tile belong to the next
sequence and must neither be stored nor leak into the last sequence's keys), short sequences,
one and several heads, the causal mask, and batches whose last sequence ends the tensor.  Every
sample of a batched launch is compared with the numpy oracle at the 1e-4 parity bound.
"""
import numpy as np
import pytest

from tests.golden.cases import A, Case
from tests.test_tensor_gemm_gpu import check_batched_per_sample

pytestmark = pytest.mark.gpu

D = 32
SHAPES = [(120, 8, 3), (128, 2, 2), (64, 1, 5), (4, 3, 2), (120, 1, 1)]  # (units, heads, batch)


def score_case(units, heads, mask):
    n = units * 3 * heads * D
    return Case(f"MHAttentionScore/{units}-{heads}-{D}/m{mask}", "MHAttentionScore",
                [A(n), A(units * heads * units, "zeros"), D, mask], (units, heads))


def out_case(units, heads):
    n = units * 3 * heads * D
    return Case(f"MHAttentionOut/{units}-{heads}-{D}", "MHAttentionOut",
                [A(units * heads * units, "unit"), A(n), A(units * heads * D, "zeros"), D], (units, heads))


@pytest.mark.parametrize("units,heads,batch", SHAPES, ids=[f"u{u}-h{h}-b{b}" for u, h, b in SHAPES])
@pytest.mark.parametrize("mask", [0, 1])
def test_score(ctx, units, heads, batch, mask):
    check_batched_per_sample(ctx, score_case(units, heads, mask), batch, 9000 + units + heads + mask)


@pytest.mark.parametrize("units,heads,batch", SHAPES, ids=[f"u{u}-h{h}-b{b}" for u, h, b in SHAPES])
def test_out(ctx, units, heads, batch):
    check_batched_per_sample(ctx, out_case(units, heads), batch, 9100 + units + heads)


def grad_case(units, heads):
    n = units * 3 * heads * D
    return Case(f"MHAttentionInsideGradients/{units}-{heads}-{D}", "MHAttentionInsideGradients",
                [A(n), A(n, "zeros"), A(units * heads * units, "unit"), A(units * heads * D, "grad")],
                (units, heads, D), meta={"softmax_scores": 1})


@pytest.mark.parametrize("units,heads,batch", SHAPES, ids=[f"u{u}-h{h}-b{b}" for u, h, b in SHAPES])
def test_inside_gradients(ctx, units, heads, batch):
    check_batched_per_sample(ctx, grad_case(units, heads), batch, 9200 + units + heads)
