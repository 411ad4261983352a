// prefill_common.cuh -- parameters shared by the two prefill implementations
// (warp-level mma.sync in fog_prefill.cu, tcgen05/TMEM in fog_prefill_tc.cu).
#pragma once

#include "fog_bias.cuh"

#include <cuda.h>
#include <stdint.h>

namespace kessie {

// Query rows are (token, head-in-group) pairs of one KV head; positions are
// absolute; the KV is paged (block_table) or dense (page coordinate = batch).
struct PrefillParams {
    const void* q; int64_t q_sb, q_st, q_sh;
    void* o; int64_t o_sb, o_st, o_sh;
    const int32_t* block_table; int64_t bt_stride;   // null: dense (page coordinate = batch)
    const int32_t* kv_lens; int kv_len_const;
    const int32_t* q_start; int q_start_const;
    int Nq, causal, window;
    const int32_t* clear_start; int clear_start_const; float fog_alpha;
    const float* fog_w; int64_t fog_w_sb;
    float scale_log2;
    int B, Hq, Hkv, G, upp, num_pages;
    FogBias bias;          // additive fog bias on the scores (vLLM path), bias.on == 0: none
    int* status;
};

// tcgen05 implementation (fog_prefill_tc.cu).  Returns kTcNotCovered when the
// shape is outside what it handles (the caller then runs the mma.sync
// kernel), else a KESSIE status.
constexpr int kTcNotCovered = 1000;
int run_prefill_tc(const PrefillParams& p, const void* q_base, const void* k_cache, const void* v_cache,
                   int64_t page_stride, int64_t token_stride, int64_t head_stride, int map_pages, int map_tokens,
                   int head_dim, bool bf16, cudaStream_t st);

}  // namespace kessie
