"""splat_b200 — the host-side mirror of instantsplat-rs's rasterizer and optimiser API
over libsplat_b200.so, the B200-native (sm_100a) differentiable Gaussian-splatting path.

    Rasterizer    instantsplat-rs/src/rasterizer.rs
    Adam          instantsplat-rs/src/optimizer.rs
    PinholeCamera instantsplat-rs/src/camera.rs
    PoseRefinement instantsplat-rs/src/pose_refinement.rs, camera_pose.rs
    Trainer       instantsplat-rs/src/training.rs (the caller of the path)
    densify       instantsplat-rs/src/densify.rs (on the device)
"""

from ._lib import SplatError, load as load_library  # noqa: F401
from .camera import PinholeCamera, cameras_extent, focal_for_fov, look_at  # noqa: F401
from .densify import (  # noqa: F401
    DENSIFY_SHORT_RUN,
    RESET_OPACITY,
    Densified,
    DensifyError,
    DensifyReport,
    DensifySettings,
    densify,
)
from .gaussians import GaussianCloud, logit, param_stride, rgb_to_sh_dc, sigmoid  # noqa: F401
from .optimizer import (  # noqa: F401
    Adam,
    LEARNING_RATES_3DGS,
    LEARNING_RATES_SHORT_RUN,
    LearningRates,
    position_rate_factor,
)
from .pose import DevicePoses, PoseCorrection, PoseRefinement, corrected_camera, pose_gradient  # noqa: F401
from .rasterizer import (  # noqa: F401
    BACKGROUND,
    Context,
    LossTerms,
    Rasterizer,
    Rendered,
    SP_BWD_ATOMIC,
    SP_BWD_DETERMINISTIC,
    SP_KEYS_FULL32,
    SP_KEYS_REF20,
    SP_TILES_ELLIPSE,
    SP_TILES_RECTANGLE,
    default_options,
)
from .training import Trainer, ground_truth_rgba  # noqa: F401,E402
