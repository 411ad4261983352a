// decode_f32.cuh -- interface between the decode entry points (fog_decode.cu)
// and the fp32 paged decode kernel (fog_decode_f32.cu).
#pragma once

#include "common.cuh"

namespace kessie {

// Arguments of one fp32 paged fog decode launch.  The workspace regions are
// the ones the bf16/fp16 decode uses (same kessie_paged_fog_decode_workspace_size):
// per-group arrival counters, then (m, l) and O/l partial slots.
struct DecodeF32Args {
    const float* q;
    int64_t q_sb, q_sh;
    const float* k_cache;
    const float* v_cache;
    int64_t page_stride, token_stride, head_stride;   // elements
    int num_pages, page_size;
    const int32_t* block_table;
    int64_t bt_stride;
    const int32_t* seq_lens;
    const int32_t* kv_off;        // nullable
    const int32_t* q_pos;         // nullable
    const int32_t* clear_start;   // nullable
    float fog_alpha;
    const float* fog_w;           // nullable
    int window;
    float sm_scale;
    int B, Hq, Hkv, D, max_seq_len;
    unsigned long long* counters; // [B*Hkv]
    uint32_t tag;                 // non-zero per-launch tag of the arrival counters
    float* part_ml;               // [slots][G][2]
    float* part_o;                // [slots][G][D]
    int slots;
    float* out;                   // rows at out + b * out_sb + h * out_sh, or null
    int64_t out_sb, out_sh;       // element strides of out per sequence and per query head
    float* out_part;              // [B][Hq][D+2] or null
    int* status;
    // Dense square attention (square_n > 0): "sequence" r of the launch is query
    // row square_row0 + r of an N = square_n token sequence -- N keys, query
    // position square_row0 + r (N - 1 when neither causal nor windowed),
    // offset 0; seq_lens, kv_off and q_pos are not read.  block_table ==
    // nullptr: page id = page index.
    int square_n;
    int square_row0;              // query row of "sequence" 0 of the launch
    int causal;
};

// Launches the fp32 decode (argument checks done by the caller).
int launch_decode_f32(const DecodeF32Args& a, cudaStream_t st);

}  // namespace kessie
