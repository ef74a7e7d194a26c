"""zenith_b200: B200-native (sm_100a) SSD chunked scan for Mamba-3, a drop-in for the
reference's ``zenith.mamba3.ssd`` behind ``Mamba3.scan``."""

from ._lib import SsdError, check_status
from .ssd import prepare_inputs, ssd, ssd_decode, ssd_dinitial_state, ssd_final_state, use_b200_scan

__all__ = ["ssd", "ssd_decode", "ssd_final_state", "ssd_dinitial_state", "use_b200_scan", "prepare_inputs", "check_status", "SsdError"]
__version__ = "0.1.0"

from .parallel import cp_ssd  # noqa: E402  (context parallelism over torch.distributed)

__all__.append("cp_ssd")

from .mamba3 import mamba3_layer_packed, mamba3_ssd_fused, use_b200_layer  # noqa: E402  (fused Mamba-3 layer body)

__all__ += ["mamba3_layer_packed", "mamba3_ssd_fused", "use_b200_layer"]

from .lm import ZenithConfig, ZenithForCausalLM, add_rmsnorm, linear_cross_entropy, train_step  # noqa: E402  (LM)

__all__ += ["ZenithConfig", "ZenithForCausalLM", "add_rmsnorm", "linear_cross_entropy", "train_step"]
