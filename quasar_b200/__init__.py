"""quasar_b200 - B200-native batched token sampler (franzvill/quasar sample.c).

The sampling work runs in libquasar_cuda.so (hand-written sm_100a kernels behind
the C ABI of include/quasar_sampler.h). Importing this package loads that
library; if it is absent the import fails - there is no CPU fallback.
"""
from ._lib import (FLAG_EXACT_SELECT, FLAG_NO_SPLIT, FLAG_NO_TMA, PATH_CANDIDATE, PATH_GREEDY, PATH_SELECT, QUASAR_NOALLOC_WORKSPACE_BYTES,
                   SYNTH_GUMBEL_PEAK, SYNTH_NORMAL, SYNTH_ZIPF, LIB_PATH, QuasarError, lib)
from .sampler import (DIAG_DTYPE, PARAMS_DTYPE, Sampler, SampleParams, make_params, params_to_device,
                      pick_batch, split_shards, synth_hist, synth_logits, synth_uniform, workspace_bytes)
from .sharded import NcclCommunicator, NcclShardedSampler, VocabShardedSampler

lib()  # fail loudly at import when the CUDA library is missing

__all__ = ["Sampler", "SampleParams", "make_params", "params_to_device", "pick_batch", "workspace_bytes", "split_shards",
           "synth_logits", "synth_hist", "synth_uniform", "PARAMS_DTYPE", "DIAG_DTYPE",
           "FLAG_EXACT_SELECT", "FLAG_NO_TMA", "FLAG_NO_SPLIT", "PATH_GREEDY", "PATH_CANDIDATE", "PATH_SELECT",
           "SYNTH_NORMAL", "SYNTH_GUMBEL_PEAK", "SYNTH_ZIPF", "LIB_PATH", "QuasarError", "lib",
           "QUASAR_NOALLOC_WORKSPACE_BYTES", "VocabShardedSampler", "NcclCommunicator", "NcclShardedSampler"]
