"""sptiles_b200 -- B200-native (sm_100a) backend for the spTiles cuda_tile workloads.

The elementwise tile add (vector_add, 1D and 2D) and the tiled mmaf matmul
(fp32 via 3xTF32, fp16, bf16, optional fused bias) run as hand-written CUDA
kernels behind the C ABI of include/sptiles_b200.h.  This package is the
Python host side: it mirrors the reference's operator API
(shaders/spirv_vector_add.py, shaders/spirv_matmul.py, shaders/matmul.py)
and its runner (shaders/spirv_runtime.py).
"""
from .api import (  # noqa: F401
    MATMUL_TILE_M, MATMUL_TILE_N, VECTOR_ADD_TILE_SIZE, cast, cutile_matmul, cutile_matmul_spirv, matmul,
    spirv_matmul, spirv_vector_add, tensor_view, vector_add, vector_fma,
)
from .runtime import (  # noqa: F401
    LOCAL_SIZE_X, ceil_div, context, context_group, device_count, grid_from_dispatch, kernel_launches, matmul_plan,
    run_tile_kernel,
    shard_range, shutdown, stream_k_split, sync, tensor_1d_descriptor, tensor_2d_descriptor, tile_raster,
)
from .module import ModuleEntry, TileModule  # noqa: F401
from ._native import DeviceAbort, NativeError, lib  # noqa: F401

__version__ = "0.1.0"
