"""Drop-in replacement for the reference ``cuda_autograd_fns`` package
(``cuda_autograd_fns/__init__.py:1-7``): the same five autograd functions, plus
``CudaLayerNorm`` over this implementation's LayerNorm kernels."""
from .cuda_causal_self_attention import CudaCausalSelfAttention
from .cuda_flash_attention import CudaFlashAttention
from .cuda_gelu_layer import CudaGeluLayer
from .cuda_layer_norm import CudaLayerNorm
from .cuda_linear_layer import CudaLinearLayer
from .cuda_softmax_layer import CudaSoftmaxLayer

__all__ = ['CudaCausalSelfAttention', 'CudaFlashAttention', 'CudaGeluLayer', 'CudaLinearLayer',
           'CudaSoftmaxLayer', 'CudaLayerNorm']
