// fog_bias.cuh -- additive fog bias of the vLLM attention path.
//
// Semantics of _FogCache._compute_into (kessie_attention.py:114-139), the bias
// the reference hands to vLLM as attn_bias, applied here inside the attention
// kernels to the scaled scores (s_j = q.k_j * sm_scale + bias_j):
//   fb = int(kv_len * (1.0 - fog_start))
//   bias_j = -fog_alpha * (1 - j / fb)^2    for 0 <= j < fb
//          = 0                              for fb <= j < kv_len
//          = recall_boost                   if j is a recalled position (overrides)
// The reference evaluates it with torch ops in the buffer dtype (the query
// dtype): arange -> divide -> rsub -> square -> scale, each result rounded to
// that dtype.  `round_mode` reproduces those roundings (0: fp32, 1: bf16,
// 2: fp16) so the bias equals the reference's buffer bit for bit.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/kessie_capi.h"

namespace kessie {

struct FogBias {
    int on;                   // 0: no additive bias
    double keep;              // 1.0 - fog_start (host-computed, as the reference's Python float)
    float neg_alpha;          // -fog_alpha
    float boost;              // recall_boost
    const uint32_t* recall;   // bitmap of recalled key positions (nullable)
    int recall_nbits;
    int round_mode;           // 0 fp32, 1 bf16, 2 fp16
};

__device__ __forceinline__ float fog_bias_round(float x, int mode) {
    if (mode == 1) return __bfloat162float(__float2bfloat16_rn(x));
    if (mode == 2) return __half2float(__float2half_rn(x));
    return x;
}

// Fog boundary of a sequence of kv_len keys: int(kv_len * (1.0 - fog_start)).
__device__ __forceinline__ int fog_bias_boundary(const FogBias& f, int kv_len) {
    return (int)((double)kv_len * f.keep);
}

// Bias of key position j (0 <= j < kv_len) for fog boundary fb.
__device__ __forceinline__ float fog_bias_at(const FogBias& f, int fb, int j) {
    float b = 0.f;
    if (j < fb) {
        const int m = f.round_mode;
        const float pos = fog_bias_round((float)j, m);
        const float t = fog_bias_round(__fdiv_rn(pos, (float)fb), m);
        float d = fog_bias_round(1.0f - t, m);
        d = fog_bias_round(d * d, m);
        b = fog_bias_round(d * f.neg_alpha, m);
    }
    if (f.recall && j < f.recall_nbits && ((__ldg(f.recall + (j >> 5)) >> (j & 31)) & 1u))
        b = fog_bias_round(f.boost, f.round_mode);
    return b;
}

// Host: validate a C-ABI bias description and convert it (null -> off).
// Returns 0 or a KESSIE status (error recorded).
int fog_bias_from_c(const kessie_fog_bias* in, FogBias* out);

}  // namespace kessie
