"""Drop-in replacement for the reference ``cuda_autograd_fns`` package
(``cuda_autograd_fns/__init__.py:1-7``): the same five autograd functions, plus
``CudaLayerNorm`` over this implementation's LayerNorm kernels, ``CudaMLP``
(fc1 -> GELU -> fc2 with the activation in the GEMM epilogues) and
``CudaLinearCrossEntropy`` (lm_head + cross entropy, chunked)."""
from .cuda_causal_self_attention import CudaCausalSelfAttention
from .cuda_flash_attention import CudaFlashAttention
from .cuda_gelu_layer import CudaGeluLayer
from .cuda_layer_norm import CudaLayerNorm
from .cuda_linear_cross_entropy import CudaLinearCrossEntropy
from .cuda_linear_layer import CudaLinearLayer
from .cuda_mlp import CudaMLP
from .cuda_softmax_layer import CudaSoftmaxLayer

__all__ = ['CudaCausalSelfAttention', 'CudaFlashAttention', 'CudaGeluLayer', 'CudaLinearLayer',
           'CudaSoftmaxLayer', 'CudaLayerNorm', 'CudaMLP', 'CudaLinearCrossEntropy']
