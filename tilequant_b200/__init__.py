"""tilequant_b200 -- B200 (sm_100a) mixed-precision 64x64 tile GEMM path.

Drop-in for the Triton path of HanzhiZhang-Ulrica/TileQuant (src/kernels/triton/,
src/kernels/quant_utils.py, src/kernels/pack.py, src/models/mixed_linear.py): the
same Python API over hand-written CUDA kernels reached through the C ABI in
``include/tilequant_b200.h`` (``libtilequant_b200.so``).
"""

from .gemm import gemm_int8_partials, gemm_mixed_fused_quant, gemm_mixed_rows_splitk, select_split_k
from .mixed_linear import (
    MixedLinear,
    MixedLinearGroup,
    MixedLinearSlice,
    fuse_projection_groups,
    reset_projection_groups,
)
from .pack import Pack, concat_packs_along_rows, is_row_major_pack, pack_weight, pack_weight_from_tile_ids
from .peer import PeerExchange, gemm_mixed_peer_sum
from .quant_utils import (
    activation_tile_absmax_scales,
    pad_to_multiple,
    quantize_activation_tile_absmax,
    quantize_activation_tile_with_scales,
)

__all__ = [
    "MixedLinear", "MixedLinearGroup", "MixedLinearSlice", "Pack", "PeerExchange", "activation_tile_absmax_scales",
    "concat_packs_along_rows", "fuse_projection_groups", "gemm_int8_partials", "gemm_mixed_fused_quant",
    "gemm_mixed_peer_sum", "gemm_mixed_rows_splitk", "is_row_major_pack", "pack_weight",
    "pack_weight_from_tile_ids", "pad_to_multiple", "quantize_activation_tile_absmax",
    "quantize_activation_tile_with_scales", "reset_projection_groups", "select_split_k",
]
