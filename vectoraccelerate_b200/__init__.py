"""vectoraccelerate_b200 -- B200-native exact flat k-NN with VectorAccelerate's kernel API.

The compute lives in ``libva_cuda.so`` (hand-written CUDA for sm_100a behind the C ABI of
``include/va_cuda.h``); this package is the host-side mirror of the reference's Swift API
(``GPUContext``, ``FusedL2TopKKernel``, ``TopKSelectionKernel``, ..., ``AcceleratedVectorIndex``).
"""

from . import _ffi
from ._ffi import (DTYPE_BF16, DTYPE_F32, INVALID_ID, METRIC_COSINE, METRIC_IP, METRIC_L2SQ, PREC_AUTO, PREC_BF16,
                   PREC_FP32, PREC_TF32)
from .context import DeviceBuffer, GPUContext, Metal4Configuration, Metal4Context, nccl_unique_id
from .errors import (BufferAllocationFailed, CollectiveFailed, ComputeFailed, InvalidInput, Timeout, Unsupported,
                     VectorError)
from .ivf import (IVFGPUIndexStructure, IVFSearchConfiguration, IVFSearchPipeline, IVFSearchResult,
                  KMeansConfiguration, KMeansPipeline, KMeansResult)
from .index import AcceleratedVectorIndex, IndexConfiguration, IndexSearchResult, SearchResults, VectorHandle
from .provider import MetalComputeProvider
from .kernels import (BinaryDatabase, BinaryQuantizationKernel, CosineSimilarityKernel, Database, DotProductKernel,
                      FusedL2TopKKernel, Int8Database, FusedL2TopKParameters, HammingDistanceKernel, L2DistanceKernel,
                      Metal4BinaryVector, Metal4FusedL2Config, Metal4FusedL2TopKResult, Metal4QuantizationResult,
                      ScalarQuantizationKernel, ShardedDatabase, TopKMergeKernel, TopKSelectionKernel,
                      WarpOptimizedSelectionKernel, knn_search_host)

# Type aliases of the reference (VectorAccelerate.swift:265-296).
L2Kernel = L2DistanceKernel
CosineKernel = CosineSimilarityKernel
DotKernel = DotProductKernel
HammingKernel = HammingDistanceKernel
TopKKernel = TopKSelectionKernel
FusedTopKKernel = FusedL2TopKKernel
ScalarQuantKernel = ScalarQuantizationKernel
BinaryQuantKernel = BinaryQuantizationKernel


def library_path() -> str:
    return _ffi.LIB_PATH


def load_library():
    """Load libva_cuda.so now (raises when it is missing)."""
    return _ffi.load()
