"""B200-native drop-in for the FasterGSVDACudaBackend operator API (FasterGSVDACudaBackend/__init__.py:14-22 of the
reference): diff_rasterize, rasterize, update_pruning_scores, RasterizerSettings, initialize_appearance,
initialize_residual_mlp, FusedAdam, update_3d_filter, relocation_adjustment and add_noise, backed by libfgs_b200.so
(hand-written sm_100a CUDA behind a C ABI)."""
from .rasterization import diff_rasterize, rasterize, update_pruning_scores, RasterizerSettings, initialize_appearance, initialize_residual_mlp
from .adam import FusedAdam
from .filter3d import update_3d_filter
from .densification import relocation_adjustment, add_noise

__all__ = [
    'diff_rasterize', 'rasterize', 'update_pruning_scores', 'RasterizerSettings', 'initialize_appearance', 'initialize_residual_mlp',
    'FusedAdam',
    'update_3d_filter',
    'relocation_adjustment', 'add_noise',
]
