"""Tensor-core linear layer (ct_linear_fwd in 3xTF32 and TF32 modes).

Covers every operand layout the linear layer's forward and backward pass to
cuda_fma (cuda_autograd_fns/cuda_linear_layer.py:11-26: x @ W with W stored
(in, out) or as weight.t(), dy @ W^T, x^T @ dy), batched weights, tile edges
in M, N and K, and reductions long enough to span several accumulation
chunks.  Reference: the FP64 product of the same FP32 inputs; error metric:
max |err| / max |ref| (test/test_linear.py:63-70 compares against nn.Linear
with atol 1e-5)."""
import pytest
import torch

import cuda_transformer_b200 as cb

from . import ct_helpers as H


def _gen(seed):
    return torch.Generator().manual_seed(seed)


def make_x(batch, m, k, mn, seed, dev):
    """x as (batch, m, k); MN-major means the m index is contiguous."""
    if mn:
        return torch.randn(batch, k, m, generator=_gen(seed)).to(dev).transpose(1, 2)
    return torch.randn(batch, m, k, generator=_gen(seed)).to(dev)


def make_w(wb, k, n, mn, seed, dev):
    """W as (wb, k, n); MN-major means the n index is contiguous."""
    if mn:
        return torch.randn(wb, k, n, generator=_gen(seed)).to(dev)
    return torch.randn(wb, n, k, generator=_gen(seed)).to(dev).transpose(1, 2)


def ref_linear(x, w, b):
    return x.double() @ w.double() + b.double()


SHAPES = [  # batch, m, k, n, w_batch
    (1, 300, 96, 200, 1),
    (3, 128, 64, 256, 3),
    (2, 260, 1100, 136, 1),   # K spans five 3xTF32 accumulation chunks, ragged M/N/K
    (1, 1024, 384, 1536, 1),  # 256-wide tiles
]


@pytest.mark.gpu
@pytest.mark.parametrize("a_mn", [False, True])
@pytest.mark.parametrize("b_mn", [False, True])
@pytest.mark.parametrize("batch,m,k,n,wb", SHAPES)
def test_layouts_3xtf32(cuda_device, a_mn, b_mn, batch, m, k, n, wb):
    x = make_x(batch, m, k, a_mn, 1, cuda_device)
    w = make_w(wb, k, n, b_mn, 2, cuda_device)
    b = torch.randn(n, generator=_gen(3)).to(cuda_device)
    out = H.linear_fwd(x, w, b, cb.PRECISION_3XTF32)
    # 3xTF32 drops lo*lo (2^-22 relative per product) and the tensor core
    # truncates its accumulator: up to ~5e-6 relative over a 256-deep chunk
    assert H.rel_err(out, ref_linear(x, w, b)) < 5e-6
    H.assert_device_clean()


@pytest.mark.gpu
@pytest.mark.parametrize("a_mn,b_mn", [(False, True), (False, False), (True, True)])
@pytest.mark.parametrize("batch,m,k,n,wb", SHAPES[:3])
def test_layouts_tf32(cuda_device, a_mn, b_mn, batch, m, k, n, wb):
    x = make_x(batch, m, k, a_mn, 4, cuda_device)
    w = make_w(wb, k, n, b_mn, 5, cuda_device)
    b = torch.randn(n, generator=_gen(6)).to(cuda_device)
    err = H.rel_err(H.linear_fwd(x, w, b, cb.PRECISION_TF32), ref_linear(x, w, b))
    # inside the TF32 band, and not FP32-exact: the tensor-core path ran
    assert 1e-6 < err < 2e-3
    H.assert_device_clean()


@pytest.mark.gpu
@pytest.mark.parametrize("workspace", [False, True])
@pytest.mark.parametrize("rows", [4096, 16384])
def test_long_reduction_weight_grad(cuda_device, rows, workspace):
    """dW = x^T dy over batch*seq rows (the linear backward's weight
    gradient), with and without the split-K schedule.  All-positive inputs
    make the accumulator's round-toward-zero bias coherent (no cancellation):
    the 256-deep chunks hold it near 5e-6 relative however long K is."""
    fin, fout = 384, 256
    g = _gen(7)
    x = torch.rand(1, rows, fin, generator=g).to(cuda_device)
    dy = torch.rand(1, rows, fout, generator=g).to(cuda_device)
    zero = torch.zeros(fout, device=cuda_device)
    dw = H.linear_fwd(x.transpose(1, 2), dy, zero, cb.PRECISION_3XTF32, workspace=workspace)
    ref = x[0].double().t() @ dy[0].double()
    assert H.rel_err(dw[0], ref) < 2e-5
    H.assert_device_clean()


@pytest.mark.gpu
@pytest.mark.parametrize("a_mn,b_mn", [(True, True), (False, True), (False, False)])
@pytest.mark.parametrize("batch,m,k,n", [(1, 384, 16384, 1536), (2, 200, 3000, 72)])
def test_split_k_matches_single_slice(cuda_device, a_mn, b_mn, batch, m, k, n):
    """The split-K schedule (few output tiles, long K) agrees with the
    one-slice schedule to rounding and is deterministic run to run."""
    x = make_x(batch, m, k, a_mn, 17, cuda_device)
    w = make_w(1, k, n, b_mn, 18, cuda_device)
    b = torch.randn(n, generator=_gen(19)).to(cuda_device)
    ref = ref_linear(x, w, b)
    o1 = H.linear_fwd(x, w, b, cb.PRECISION_3XTF32, workspace=True)
    o2 = H.linear_fwd(x, w, b, cb.PRECISION_3XTF32, workspace=True)
    o0 = H.linear_fwd(x, w, b, cb.PRECISION_3XTF32, workspace=False)
    assert torch.equal(o1, o2)
    assert H.rel_err(o1, ref) < 5e-6 and H.rel_err(o0, ref) < 5e-6
    H.assert_device_clean()


@pytest.mark.gpu
def test_strided_bias_and_batched_weights(cuda_device):
    batch, m, k, n = 2, 200, 128, 96
    x = make_x(batch, m, k, False, 8, cuda_device)
    w = make_w(batch, k, n, True, 9, cuda_device)
    b = torch.randn(2 * n, generator=_gen(10)).to(cuda_device)[::2]
    out = H.linear_fwd(x, w, b, cb.PRECISION_3XTF32)
    assert H.rel_err(out, ref_linear(x, w, b)) < 5e-6
    H.assert_device_clean()


@pytest.mark.gpu
def test_deterministic(cuda_device):
    x = make_x(1, 2048, 1536, False, 11, cuda_device)
    w = make_w(1, 1536, 384, True, 12, cuda_device)
    b = torch.randn(384, generator=_gen(13)).to(cuda_device)
    o1 = H.linear_fwd(x, w, b)
    o2 = H.linear_fwd(x, w, b)
    assert torch.equal(o1, o2)


@pytest.mark.gpu
def test_unaligned_strides_fall_back(cuda_device):
    """K = 70 rows are not 16-byte aligned: served by the CUDA-core kernel,
    same results."""
    x = make_x(1, 512, 70, False, 14, cuda_device)
    w = make_w(1, 70, 120, True, 15, cuda_device)
    b = torch.randn(120, generator=_gen(16)).to(cuda_device)
    out = H.linear_fwd(x, w, b, cb.PRECISION_3XTF32)
    assert H.rel_err(out, ref_linear(x, w, b)) < 1e-6


@pytest.mark.gpu
@pytest.mark.parametrize("workspace", [False, True])
@pytest.mark.parametrize("batch,m,k,n", [(1, 300, 96, 118), (2, 200, 3000, 70)])
def test_output_rows_not_16_byte_aligned(cuda_device, workspace, batch, m, k, n):
    """n not a multiple of 4: the output rows cannot be TMA-stored, so the
    epilogue writes rows per thread (x and W^T still arrive by TMA)."""
    x = make_x(batch, m, k, False, 20, cuda_device)
    w = make_w(1, k, n, False, 21, cuda_device)
    b = torch.randn(n, generator=_gen(22)).to(cuda_device)
    out = H.linear_fwd(x, w, b, cb.PRECISION_3XTF32, workspace=workspace)
    assert H.rel_err(out, ref_linear(x, w, b)) < 5e-6
    H.assert_device_clean()
