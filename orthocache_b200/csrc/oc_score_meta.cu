// The fused decode layer with its block decisions taken from write-time
// spectral metadata (score_tma_kernel<128, true, true>), compiled as a unit
// of its own: the kernel template and its helpers come from oc_score.cu, and
// nothing of that file's host interface is defined here except
// decode_fused_meta and this unit's status and wait-limit hooks.  Keeping the
// two instantiations in separate units keeps the key-scoring layer's code
// generation independent of this one.
#define OC_SCORE_META_TU 1
#include "oc_score.cu"
