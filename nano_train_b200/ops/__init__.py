"""Hot ops of nano_train_b200: sm_100a kernels behind autograd functions."""
from ._ext import available, check_status, ext  # noqa: F401
from .activation import gelu, swiglu  # noqa: F401
from .embedding import embedding  # noqa: F401
from .linear import gemm, linear  # noqa: F401
from .loss import cross_entropy  # noqa: F401
from .norm import add_rms_norm, layer_norm, rms_norm  # noqa: F401
from .optim import adamw_flat_, grad_stats_  # noqa: F401
from .rope import apply_rope  # noqa: F401
