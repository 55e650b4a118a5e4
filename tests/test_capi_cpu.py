"""CPU tests of the boundary: the C-ABI library loads and exports every symbol
include/ct_b200.h declares; the torch extension registers the reference's
operator schemas verbatim; fake (meta) kernels give the reference's shapes.
No compute is launched (no GPU here)."""
import ctypes
import re

import pytest
import torch

import cuda_transformer_b200 as cb

from .conftest import ROOT

REFERENCE_SCHEMAS = {
    # Transformer_launchers/*.cu m.def(...) strings
    "cuda_fma": "cuda_fma(Tensor x, Tensor weights, Tensor bias) -> Tensor",
    "db_calculation": "db_calculation(Tensor dy) -> Tensor",
    "cuda_softmax": "cuda_softmax(Tensor x) -> Tensor",
    "cuda_softmax_bwd": "cuda_softmax_bwd(Tensor probs, Tensor dp) -> Tensor",
    "gelu_activation": "gelu_activation(Tensor x) -> Tensor",
    "gelu_activation_bwd": "gelu_activation_bwd(Tensor x, Tensor dy) -> Tensor",
    "flash_attention_fwd":
        "flash_attention_fwd(Tensor Q, Tensor K, Tensor V, bool causal) -> (Tensor, Tensor)",
    "flash_attention_bwd":
        "flash_attention_bwd(Tensor Q, Tensor K, Tensor V, Tensor O, Tensor dO, Tensor L, "
        "bool causal) -> (Tensor, Tensor, Tensor)",
    "causal_self_attention_fwd":
        "causal_self_attention_fwd(Tensor qkv, int nh, bool causal) -> (Tensor, Tensor)",
    "causal_self_attention_bwd":
        "causal_self_attention_bwd(Tensor Q, Tensor K, Tensor V, Tensor probs, Tensor dO) -> "
        "(Tensor, Tensor, Tensor)",
}


def declared_symbols():
    text = (ROOT / "include" / "ct_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ct_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = cb.lib()
    syms = declared_symbols()
    assert len(syms) >= 20
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in ct_b200.h but not exported"
    assert set(syms) == set(cb.SIGNATURES), "ctypes signature table out of sync with the header"


def test_test_only_diagnostics_stay_out_of_the_product():
    """Layout checks and the throughput probe live in tests/diag/libct_diag.so,
    which exports what its header declares; the product library exports none
    of them."""
    from tests import diag

    text = re.sub(r"/\*.*?\*/", "", diag.HEADER_PATH.read_text(), flags=re.S)
    syms = sorted(set(re.findall(r"\b(ct_[a-z0-9_]+)\s*\(", text)))
    assert syms == sorted(diag.SIGNATURES)
    dl = diag.lib()
    for s in syms:
        assert hasattr(dl, s), s
        assert not hasattr(cb.lib(), s), f"{s} is exported by the product library"


def test_status_strings_and_version():
    lib = cb.lib()
    assert lib.ct_version() >= 10000
    assert cb.status_string(cb.CT_ERR_UNSUPPORTED_HEAD_DIM).startswith("Unsupported head dimension")
    for rc in range(0, 9):
        assert cb.status_string(rc)


def test_workspace_queries():
    lib = cb.lib()
    # delta, then the one-kernel backward's ordering counters (4 per 64-query
    # tile) and one ticket per 4096-long segment
    assert lib.ct_fa2_bwd_workspace_size(4, 32, 4096, 64) == 4 * 32 * 4096 * 4 + (128 * 64 * 4 + 1) * 4
    assert lib.ct_fa2_bwd_workspace_size(1, 1, 8193, 64) == 33024 + (129 * 4 + 3) * 4
    assert lib.ct_fa2_bwd_workspace_size(-1, 1, 1, 64) == 0
    assert lib.ct_bias_grad_workspace_size(1, 16384, 1536) >= 1536 * 4
    assert lib.ct_layernorm_bwd_workspace_size(16384, 384) >= 2 * 384 * 4


def test_invalid_arguments_rejected_before_any_device_work():
    lib = cb.lib()
    s = (ctypes.c_int64 * 4)(1, 1, 1, 1)
    # head_dim 48 is unsupported: rejected during validation
    rc = lib.ct_fa2_fwd(None, s, None, s, None, s, None, None, 1, 1, 8, 48, 0, 0, None)
    assert rc == cb.CT_ERR_UNSUPPORTED_HEAD_DIM
    rc = lib.ct_fa2_fwd(None, s, None, s, None, s, None, None, -1, 1, 8, 64, 0, 0, None)
    assert rc == cb.CT_ERR_INVALID_ARGUMENT
    rc = lib.ct_fa2_fwd(None, s, None, s, None, s, None, None, 1, 1, 8, 64, 0, 7, None)
    assert rc == cb.CT_ERR_INVALID_ARGUMENT
    # B*H is bounded factor by factor, so a product that would wrap is rejected
    for B, Hh in ((2 ** 62 + 1, 4), (2 ** 40, 2 ** 40), (2 ** 31, 1)):
        rc = lib.ct_fa2_fwd(None, s, None, s, None, s, None, None, B, Hh, 1, 64, 0, 0, None)
        assert rc == cb.CT_ERR_INVALID_ARGUMENT, (B, Hh)
    # fused linear options: a GELU epilogue needs its output, accumulate goes
    # with no epilogue, column sums need batch 1
    s3 = (ctypes.c_int64 * 3)(1, 1, 1)
    p = ctypes.c_void_p(256)
    assert lib.ct_linear_fwd_ex(p, s3, p, s3, p, 1, p, 1, 4, 4, 4, 1, 0, 1, None, None, None, 0,
                                None, 0, None) == cb.CT_ERR_INVALID_ARGUMENT
    assert lib.ct_linear_fwd_ex(p, s3, p, s3, p, 1, p, 1, 4, 4, 4, 1, 0, 2, None, None, None, 0,
                                None, 0, None) == cb.CT_ERR_INVALID_ARGUMENT
    assert lib.ct_linear_fwd_ex(p, s3, p, s3, p, 1, p, 1, 4, 4, 4, 1, 0, 1, p, None, None, 1,
                                None, 0, None) == cb.CT_ERR_INVALID_ARGUMENT
    assert lib.ct_linear_fwd_ex(p, s3, p, s3, p, 1, p, 2, 4, 4, 4, 1, 0, 0, None, None, p, 0,
                                None, 0, None) == cb.CT_ERR_INVALID_ARGUMENT
    assert lib.ct_linear_fwd_ex(p, s3, p, s3, p, 1, p, 1, 4, 4, 4, 1, 0, 3, None, None, None, 0,
                                None, 0, None) == cb.CT_ERR_INVALID_ARGUMENT
    assert lib.ct_cross_entropy_fwd_bwd(p, 4, 2, 8, p, -100, p, None) == cb.CT_ERR_INVALID_ARGUMENT
    # the one-kernel backward covers TF32 at head dim 64 only
    s3b = (ctypes.c_int64 * 3)(1, 1, 1)
    for D, prec, want in ((32, cb.PRECISION_TF32, cb.CT_ERR_UNSUPPORTED_HEAD_DIM),
                          (64, cb.PRECISION_3XTF32, cb.CT_ERR_INVALID_ARGUMENT),
                          (64, cb.PRECISION_FP32, cb.CT_ERR_INVALID_ARGUMENT)):
        rc = lib.ct_fa2_bwd_fused(p, s, p, s, p, s, p, s, p, s, p, s3b, p, p, p, p, 1 << 20,
                                  1, 1, 64, D, 1, prec, None)
        assert rc == want, (D, prec, rc)
    # LayerNorm rows are at most 8192 wide
    rc = lib.ct_layernorm_fwd(None, None, None, None, None, None, 1, 8193, ctypes.c_float(1e-5), None)
    assert rc == cb.CT_ERR_INVALID_ARGUMENT
    rc = lib.ct_layernorm_bwd(None, None, None, None, None, None, None, None, 1, 8193, None, 0, None)
    assert rc == cb.CT_ERR_INVALID_ARGUMENT


def test_torch_schemas_match_reference():
    import cuda_transformer  # noqa: F401  (loads _C)
    for name, schema in REFERENCE_SCHEMAS.items():
        op = getattr(torch.ops.cuda_transformer, name).default
        assert str(op._schema) == "cuda_transformer::" + schema


def test_ops_module_surface():
    from cuda_transformer import ops
    for name in ["cuda_fma", "db_calculation", "cuda_softmax", "cuda_softmax_bwd",
                 "gelu_activation", "gelu_activation_bwd", "causal_self_attention_fwd",
                 "causal_self_attention_bwd", "flash_attention_fwd", "flash_attention_bwd"]:
        assert callable(getattr(ops, name)) and name in ops.__all__
    import cuda_autograd_fns
    for name in ['CudaCausalSelfAttention', 'CudaFlashAttention', 'CudaGeluLayer',
                 'CudaLinearLayer', 'CudaSoftmaxLayer']:
        assert issubclass(getattr(cuda_autograd_fns, name), torch.autograd.Function)


def test_fake_kernels_give_reference_shapes():
    from torch._subclasses.fake_tensor import FakeTensorMode
    from cuda_transformer import ops
    with FakeTensorMode():
        q = torch.empty(2, 4, 33, 64)
        o, l = ops.flash_attention_fwd(q, q, q, True)
        assert o.shape == (2, 4, 33, 64) and l.shape == (2, 4, 33)
        dq, dk, dv = ops.flash_attention_bwd(q, q, q, o, o, l, True)
        assert dq.shape == q.shape and dk.shape == q.shape and dv.shape == q.shape
        x = torch.empty(3, 5, 7)
        w = torch.empty(7, 11)
        assert ops.cuda_fma(x, w, torch.empty(11)).shape == (3, 5, 11)
        assert ops.db_calculation(torch.empty(3, 5, 11)).shape == (11,)
        y, m, r = ops.layernorm_fwd(torch.empty(6, 384), torch.empty(384), torch.empty(384))
        assert y.shape == (6, 384) and m.shape == (6,) and r.shape == (6,)
        o, a, cs = ops.linear_fused(x, w, torch.empty(11), 0, ops.EPILOGUE_GELU, None, False)
        assert o.shape == (3, 5, 11) and a.shape == (3, 5, 11) and cs.numel() == 0
        o, a, cs = ops.linear_fused(x[:1], w, torch.empty(11), 0, 0, None, True)
        assert cs.shape == (11,) and a.numel() == 0
        assert ops.cross_entropy_fwd_bwd_(torch.empty(4, 9), torch.empty(4, dtype=torch.long)).shape == (4,)


def test_product_path_does_not_import_oracle():
    for pkg in ("cuda_transformer", "cuda_autograd_fns", "cuda_transformer_b200"):
        for f in (ROOT / pkg).rglob("*.py"):
            src = f.read_text()
            assert "import oracle" not in src and "from oracle" not in src, f
