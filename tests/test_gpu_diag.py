"""On-device checks of the tensor-core operand layouts the kernels rely on
(K-major / MN-major shared-memory operands in the 128-byte swizzle, A from
Tensor Memory) and of how the tensor core treats the low mantissa bits of an
FP32 operand: it truncates them, which the 3xTF32 split relies on (a raw FP32
tile in shared memory is read as its truncated "hi" part)."""
import pytest
import torch

from . import ct_helpers as H

MODES = {0: "ss_kk", 1: "ss_k_mn", 2: "ts_k", 3: "ts_mn", 4: "ss_mn_mn"}


def _tf32_exact(shape, gen, device):
    x = torch.randn(*shape, generator=gen, dtype=torch.float32)
    x = (x.view(torch.int32) & ~0x1FFF).view(torch.float32)  # low 13 bits zero: exact in TF32
    return x.to(device)


@pytest.mark.gpu
@pytest.mark.parametrize("mode", sorted(MODES))
@pytest.mark.parametrize("n", [32, 64, 128])
def test_umma_layouts(cuda_device, mode, n):
    g = torch.Generator().manual_seed(100 + 10 * mode + n)
    if mode == 4:
        a = _tf32_exact((32, 128), g, cuda_device)      # [k][m]
        amat = a.t()
    else:
        a = _tf32_exact((128, 32), g, cuda_device)      # [m][k]
        amat = a
    if mode in (1, 3, 4):
        b = _tf32_exact((32, n), g, cuda_device)        # [k][n]
        bmat = b
    else:
        b = _tf32_exact((n, 32), g, cuda_device)        # [n][k]
        bmat = b.t()
    d = H.diag_umma(mode, a.contiguous(), b.contiguous(), n)
    ref = amat.double() @ bmat.double()
    assert H.rel_err(d, ref) < 1e-6, MODES[mode]
    H.assert_device_clean()


@pytest.mark.gpu
def test_tf32_operand_rounding_rule(cuda_device, record_property):
    """A holds values whose 13 low mantissa bits are set; B is the identity, so
    D shows the TF32 value the tensor core used for each A element."""
    base = torch.linspace(1.0, 2.0, 128 * 32).reshape(128, 32)
    bits = base.view(torch.int32) | 0x1FFF | 0x1000  # above the half-way point of a TF32 ulp
    a = bits.view(torch.float32).contiguous()
    b = torch.zeros(32, 32)
    b.fill_diagonal_(1.0)
    d = H.diag_umma(0, a.to(cuda_device), b.to(cuda_device), 32).cpu()
    trunc = (a.view(torch.int32) & ~0x1FFF).view(torch.float32)
    is_trunc = torch.equal(d, trunc)
    is_round = torch.equal(d, (trunc.double() + 2.0 ** -10 * 2.0 ** torch.floor(torch.log2(trunc.double()))).float())
    record_property("tf32_operand_rule", "truncate" if is_trunc else ("round" if is_round else "other"))
    print("tf32 operand rule:", "truncate" if is_trunc else ("round" if is_round else "other"))
    assert is_trunc, "3xTF32 split assumes the tensor core truncates FP32 operands to TF32"
    H.assert_device_clean()


@pytest.mark.gpu
def test_mma_rate_probe_runs(cuda_device):
    """The test-only tensor-pipe probe completes on every SM and wider N never
    costs fewer cycles per MMA than narrower N."""
    from tests import diag

    L = diag.lib()
    sms = torch.cuda.get_device_properties(cuda_device).multi_processor_count
    cyc = torch.zeros(sms, dtype=torch.int64, device=cuda_device)
    per = {}
    for n in (32, 128):
        diag.check(L.ct_diag_mma_rate(n, 1, 200, sms, H._p(cyc), H._stream()), "rate")
        torch.cuda.synchronize()
        assert bool((cyc > 0).all())
        per[n] = cyc.double().mean().item() / 800
    assert per[128] >= per[32] * 0.95
    # every operand form and the two-issuer variant complete (flags: A in TMEM,
    # B MN-major, two issuing threads); out-of-range flags are rejected
    for flags in (0, 2, 3, 5, 7):
        diag.check(L.ct_diag_mma_rate(64, flags, 50, sms, H._p(cyc), H._stream()), "rate")
        torch.cuda.synchronize()
        assert bool((cyc > 0).all()), flags
    assert L.ct_diag_mma_rate(256, 4, 50, sms, H._p(cyc), H._stream()) != 0
    assert L.ct_diag_mma_rate(64, 8, 50, sms, H._p(cyc), H._stream()) != 0
    assert diag.status() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("mode", [m for m in range(16) if not (m & 8 and m & 1)])
@pytest.mark.parametrize("n", [32, 64])
def test_umma_m64_layouts(cuda_device, mode, n):
    """M = 64 MMAs: rows in lanes 32*(r//16) + r%16 (+16 for the upper half of
    each lane quadrant), A from shared memory (K-major, or MN-major together
    with an MN-major B: the fused backward's dQ product) or TMEM, D read with
    the 32x32b or the 16-lane 16x32bx2 shape."""
    from tests import diag

    if (mode & 4) and n != 32:
        pytest.skip("16x32bx2 read covers n = 32")
    g = torch.Generator().manual_seed(300 + 10 * mode + n)
    a = _tf32_exact((64, 32), g, cuda_device)
    b = _tf32_exact((n, 32), g, cuda_device)
    d = torch.full((64, n), float("nan"), device=cuda_device)
    aa, bb = (a.t().contiguous(), b.t().contiguous()) if mode & 8 else (a, b)
    diag.check(diag.lib().ct_diag_umma_m64(mode, H._p(aa), H._p(bb), H._p(d), n, H._stream()),
               "ct_diag_umma_m64")
    torch.cuda.synchronize()
    assert diag.status() == 0
    ref = a.double() @ b.double().t()
    assert H.rel_err(d, ref) < 1e-6, mode


@pytest.mark.gpu
@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("n", [64, 128])
def test_umma_pair_layouts(cuda_device, mode, n):
    """CTA pair (cta_group::2, M = 256): each CTA holds 128 rows of A and D in
    its own Tensor Memory and half of B's N rows in its shared memory (K-major
    or MN-major); the odd CTA's readiness reaches the issuing even CTA by a
    remote barrier arrival and the commit completes both CTAs' barriers."""
    from tests import diag

    g = torch.Generator().manual_seed(500 + 10 * mode + n)
    a = _tf32_exact((256, 64), g, cuda_device)
    b = _tf32_exact((n, 64), g, cuda_device)  # [n][k]
    d = torch.full((256, n), float("nan"), device=cuda_device)
    bb = b.t().contiguous() if mode == 1 else b
    diag.check(diag.lib().ct_diag_umma_pair(mode, H._p(a), H._p(bb), H._p(d), n, H._stream()),
               "ct_diag_umma_pair")
    torch.cuda.synchronize()
    assert diag.status() == 0
    ref = a.double() @ b.double().t()
    assert H.rel_err(d, ref) < 1e-6, mode
