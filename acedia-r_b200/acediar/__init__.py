"""acediar — B200 kernels for acediaR's data-parallel tensor path.

The compute lives in libacediar_b200.so (CUDA, sm_100a) behind the C ABI of
include/acd.h; this package is the host-side mirror of the R gpuTensor API.
"""
from ._lib import AcdError, lib  # noqa: F401
from .tensor import (  # noqa: F401
    abs, argmax, argmin, as_array, as_tensor, ceiling, check_device_status, compare, contiguous, context, cos,
    cumprod, cumsum, dtype, empty_tensor, erf, exp, floor, from_torch, fused, gpu_tensor, gpuTensor, is_contiguous,
    log, max, mean, min, permute_view, pmax, pmin, prod, relu, reshape, round, shape, sigmoid, sin, softmax, sqrt,
    sum, sum_var, synchronize, tanh, tensor_count, tensor_max, tensor_mean, tensor_min, tensor_prod, tensor_sum,
    tensor_var, to_dtype, transpose, transpose_view, var, view, which_max, which_min, subset, assign, concat,
    concat_tensor, stack, stack_tensor, repeat_tensor, pad, pad_tensor, set_seed, rand_tensor, rnorm_tensor,
    rand_tensor_uniform, rand_tensor_normal, runif, rnorm, any, all, diff, range_, is_finite, create_ones_like, all_equal,
    tensor_pow, permute, size, dim, as_vector, as_numeric, to_numeric, tensor_to_scalar, shares_memory, tensor_info,
    set_random_seed, gpu_available, gpu_info, gpu_memory_available, gpu_status, gpu_add, gpu_multiply, gpu_scale, gpu_dot)
