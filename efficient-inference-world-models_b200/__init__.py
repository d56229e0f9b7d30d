"""B200-native Oasis-500M DiT denoising forward (sm_100a), a drop-in for the
worldserve hot path: ``dit(x, t, external_cond)`` plus the sampler and KV-cache
interfaces around it.  All compute runs in ``liboasis_b200.so`` (C ABI in
``include/oasis_b200.h``); there is no CPU fallback.
"""

from . import _native
from ._native import OasisError, lib, version
from .dit import OasisDiTB200
from .kv_cache import KVCacheB200, attn_spatial, attn_temporal
from .manager import KVCacheManagerB200, ProgressiveKVQuantizerB200, RollingKVCacheB200
from .oasis import (action_step_schedule, alphas_cumprod, generate, rollout_dpmpp,
                    sigmoid_beta_schedule, steps_for_action_magnitude)
from .samplers import DPMSolverPPSampler, ddim_update, dpmpp2m_update
from .vae import OasisVAEDecoderB200, random_vae_state_dict, vae_param_shapes
from .weights import pack_weights, param_shapes, random_state_dict, rope_tables

__all__ = [
    "OasisDiTB200", "OasisVAEDecoderB200", "KVCacheB200", "KVCacheManagerB200", "ProgressiveKVQuantizerB200",
    "RollingKVCacheB200",
    "DPMSolverPPSampler", "OasisError", "action_step_schedule", "alphas_cumprod", "attn_spatial", "attn_temporal",
    "ddim_update", "dpmpp2m_update", "generate", "lib", "pack_weights", "param_shapes",
    "random_state_dict", "random_vae_state_dict", "rollout_dpmpp", "rope_tables", "sigmoid_beta_schedule", "steps_for_action_magnitude", "vae_param_shapes", "version",
]
