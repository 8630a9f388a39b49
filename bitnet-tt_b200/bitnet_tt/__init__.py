"""bitnet_tt (B200 build): the packed-ternary BitLinear decode path of
deveworld/bitnet-tt, re-implemented on hand-written sm_100a CUDA kernels.

The Python API keeps the reference's module layout and call sites
(layers.bitlinear.Linear, model.bitnet.create_model, utils.weights,
inference.generator_batch32.Batch32Generator); the compute runs in
libbitnet_b200.so through the C ABI declared in include/bitnet_b200.h.
"""

__version__ = "0.1.0"

from .config import BitNet2B4TConfig, BitNetConfig, BitNetMiniConfig, get_config  # noqa: F401
