"""B200-native routed micro-expert channel mixer for SPALMER.

Drop-in for ``spalmer.experts.MicroExpertChannelMixer`` (same constructor,
``forward`` contract and ``state_dict``), executed by hand-written sm_100a
kernels in ``libspx`` (``include/spx.h``).
"""

from spalmer_b200.config import MicroExpertsConfig
from spalmer_b200.experts import (
    B200ChannelBlock,
    B200MicroExpertChannelMixer,
    ChannelMixerOutput,
    ExpertPotentiationController,
    ExpertResidency,
    MicroExpertBank,
    MicroExpertChannelMixer,
    NativeExpertPrecisionError,
    RMSNorm,
    SurpriseRouter,
    SwiGLU,
    dispatch,
    rms_norm,
    route,
)

__all__ = [
    "B200ChannelBlock",
    "B200MicroExpertChannelMixer",
    "ChannelMixerOutput",
    "ExpertPotentiationController",
    "ExpertResidency",
    "MicroExpertBank",
    "MicroExpertChannelMixer",
    "MicroExpertsConfig",
    "NativeExpertPrecisionError",
    "RMSNorm",
    "SurpriseRouter",
    "SwiGLU",
    "dispatch",
    "rms_norm",
    "route",
]
