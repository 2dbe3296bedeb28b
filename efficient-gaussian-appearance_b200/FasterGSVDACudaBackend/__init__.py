"""B200-native drop-in for the FasterGSVDACudaBackend operator API (FasterGSVDACudaBackend/__init__.py:14-22 of the
reference): diff_rasterize, rasterize, update_pruning_scores, RasterizerSettings, initialize_appearance,
initialize_residual_mlp and FusedAdam, backed by libfgs_b200.so (hand-written sm_100a CUDA behind a C ABI)."""
from .rasterization import diff_rasterize, rasterize, update_pruning_scores, RasterizerSettings, initialize_appearance, initialize_residual_mlp
from .adam import FusedAdam

__all__ = [
    'diff_rasterize', 'rasterize', 'update_pruning_scores', 'RasterizerSettings', 'initialize_appearance', 'initialize_residual_mlp',
    'FusedAdam',
]
