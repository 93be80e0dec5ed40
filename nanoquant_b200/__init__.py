"""nanoquant_b200: NanoQuant's packed binary low-rank linear, built for B200 (sm_100a).

The public surface mirrors the packed-linear operator of NanoQuant's
deployment runtime (``nanoquant.runtime``): the backend contract types, packed
layout v1 and its layer state, the product-codebook state, and
:class:`CudaPackedSm100Backend`, whose arithmetic runs in the C-ABI library
``libnqb.so`` (``include/nqb.h``).
"""

from nanoquant_b200.backend import (
    BackendCapabilities,
    PreparedLayer,
    ProjectionMemberSpec,
    QuantizedLinearSpec,
    RuntimeBackend,
    SupportResult,
    WorkloadSpec,
    evaluate_capabilities,
)
from nanoquant_b200.cuda_backend import (
    CUDA_SM100_BACKEND_NAME,
    CUDA_SM100_BACKEND_VERSION,
    CudaPackedSm100Backend,
    Sm100ProjectionGroup,
    grouped_cuda_projection,
    grouped_sm100_projection,
    prepare_cuda_projection_group,
    prepare_sm100_projection_group,
)
from nanoquant_b200.logical import LogicalLayerState, canonical_torch_dtype, parse_torch_dtype
from nanoquant_b200.overlay import OutlierRowOverlay, OverlaidLayerState
from nanoquant_b200.packed import (
    GGUF_TENSOR_SUFFIXES,
    PACKED_LAYOUT_VERSION,
    PACKED_TENSOR_NAMESPACE,
    PACKED_WORD_BITS,
    PackedLayerState,
    PackedLayoutMetadata,
    pack_logical_layer,
    pack_sign_matrix,
    packed_row_stride_bytes,
    packed_word_count,
    supports_vector_word_loads,
    unpack_sign_matrix,
)
from nanoquant_b200.artifact import (
    OpenPackedArtifact,
    PackedArtifactError,
    open_packed_artifact,
)
from nanoquant_b200.mixed_v import (
    MIXED_V_FORMAT_VERSION,
    MixedVLayerState,
    decode_mixed_v_right_words,
    mixed_v_correction_pair_table,
    mixed_v_from_packed_words,
    mixed_v_payload_word_count,
    pack_mixed_v_records,
    unpack_mixed_v_records,
)
from nanoquant_b200.product_codebook import (
    PRODUCT_CODEBOOK_FORMAT_VERSION,
    ProductCodebookLayerState,
    decode_product_codebook_right_words,
    pack_product_codebook_indices,
    pack_product_half_table,
    product_codebook_payload_word_count,
    unpack_product_codebook_indices,
    unpack_product_half_table,
)

__all__ = [
    "OpenPackedArtifact",
    "PackedArtifactError",
    "open_packed_artifact",
    "MIXED_V_FORMAT_VERSION",
    "MixedVLayerState",
    "decode_mixed_v_right_words",
    "mixed_v_correction_pair_table",
    "mixed_v_from_packed_words",
    "mixed_v_payload_word_count",
    "pack_mixed_v_records",
    "unpack_mixed_v_records",
    "BackendCapabilities",
    "CUDA_SM100_BACKEND_NAME",
    "CUDA_SM100_BACKEND_VERSION",
    "CudaPackedSm100Backend",
    "GGUF_TENSOR_SUFFIXES",
    "LogicalLayerState",
    "OutlierRowOverlay",
    "OverlaidLayerState",
    "PACKED_LAYOUT_VERSION",
    "PACKED_TENSOR_NAMESPACE",
    "PACKED_WORD_BITS",
    "PRODUCT_CODEBOOK_FORMAT_VERSION",
    "PackedLayerState",
    "PackedLayoutMetadata",
    "PreparedLayer",
    "ProductCodebookLayerState",
    "ProjectionMemberSpec",
    "QuantizedLinearSpec",
    "RuntimeBackend",
    "Sm100ProjectionGroup",
    "SupportResult",
    "WorkloadSpec",
    "canonical_torch_dtype",
    "decode_product_codebook_right_words",
    "evaluate_capabilities",
    "grouped_cuda_projection",
    "grouped_sm100_projection",
    "pack_logical_layer",
    "pack_product_codebook_indices",
    "pack_product_half_table",
    "pack_sign_matrix",
    "packed_row_stride_bytes",
    "packed_word_count",
    "parse_torch_dtype",
    "prepare_cuda_projection_group",
    "prepare_sm100_projection_group",
    "product_codebook_payload_word_count",
    "supports_vector_word_loads",
    "unpack_product_codebook_indices",
    "unpack_product_half_table",
    "unpack_sign_matrix",
]
