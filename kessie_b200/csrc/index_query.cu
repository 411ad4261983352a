// index_query.cu -- cosine similarity of one query against a conversation
// index, with the top-k rows selected on the device.
//
// Semantics of _kessie_index_query_kernel (kessie_hip_kernels.py:343-360):
//   qn = q / sqrt(sum(q^2) + 1e-8)
//   sim_i = sum(qn * x_i / sqrt(sum(x_i^2) + 1e-8))      (normalize_rows = 1)
//   sim_i = sum(qn * x_i)                                 (rows stored normalised,
//                                                          as VectorIndex keeps them,
//                                                          kessie_exp3.py:69-81)
// top-k: the k largest sims, descending, ties to the lower row index.
//
// Design (B200, HBM-bound: N * dim * 4 bytes per query): one warp per row
// (each lane reads 16-byte chunks of the row, four rows in flight per warp),
// a warp-wide reduction gives the row's dot product and squared norm; every
// warp keeps its running top-k in registers (lane s holds rank s) and inserts
// each row with one ballot + shuffle; the CTA merges its warps' lists in
// shared memory and writes one list per CTA; a one-CTA second launch merges
// the CTA lists.
#include "common.cuh"

#include <float.h>

namespace kessie {
namespace {

constexpr int kIqWarps = 8;
constexpr int kIqThreads = kIqWarps * 32;
constexpr int kIqMaxK = 32;
constexpr int kIqMergeThreads = 1024;

// (score, index) order: higher score first, lower index first on ties.
__device__ __forceinline__ bool iq_better(float a, int ia, float b, int ib) {
    return a > b || (a == b && ia < ib);
}

// Warp-register top-k: lane s < k holds rank s.  Inserts (v, iv) (warp-uniform).
__device__ __forceinline__ void iq_insert(float& val, int& idx, int k, float v, int iv, int lane) {
    const float last = __shfl_sync(0xffffffffu, val, k - 1);
    const int last_i = __shfl_sync(0xffffffffu, idx, k - 1);
    if (!iq_better(v, iv, last, last_i)) return;
    // rank of the newcomer = number of entries better than it
    const unsigned better = __ballot_sync(0xffffffffu, lane < k && iq_better(val, idx, v, iv));
    const int pos = __popc(better);
    const float up_v = __shfl_up_sync(0xffffffffu, val, 1);
    const int up_i = __shfl_up_sync(0xffffffffu, idx, 1);
    if (lane < k) {
        if (lane > pos) { val = up_v; idx = up_i; }
        else if (lane == pos) { val = v; idx = iv; }
    }
}

__device__ __forceinline__ float iq_warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Pass 1: similarities (optional output) and one top-k list per CTA.
__global__ void __launch_bounds__(kIqThreads) index_query_kernel(const float* __restrict__ query,
                                                                 const float* __restrict__ index, int n, int dim,
                                                                 int normalize_rows, float* __restrict__ sims,
                                                                 int k, float* __restrict__ cand_val,
                                                                 int* __restrict__ cand_idx) {
    __shared__ float s_val[kIqWarps][kIqMaxK];
    __shared__ int s_idx[kIqWarps][kIqMaxK];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int d4 = dim >> 2;                               // 16-byte chunks per row
    // query norm (every warp computes it; dim is small)
    float qq = 0.f;
    for (int c = lane; c < d4; c += 32) {
        const float4 x = __ldg(reinterpret_cast<const float4*>(query) + c);
        qq += x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
    }
    const float qinv = 1.f / sqrtf(iq_warp_sum(qq) + 1e-8f);
    float val = -FLT_MAX;
    int idx = INT_MAX;
    const int gw = blockIdx.x * kIqWarps + warp, nw = gridDim.x * kIqWarps;
    constexpr int R = 4;                                   // rows in flight per warp
    for (int r0 = gw * R; r0 < n; r0 += nw * R) {
        float dot[R], sq[R];
#pragma unroll
        for (int u = 0; u < R; ++u) { dot[u] = 0.f; sq[u] = 0.f; }
        for (int c = lane; c < d4; c += 32) {
            const float4 qv = __ldg(reinterpret_cast<const float4*>(query) + c);
            float4 x[R];
#pragma unroll
            for (int u = 0; u < R; ++u) {
                const int r = r0 + u;
                x[u] = r < n ? ldg_stream_f4(index + (size_t)r * dim + 4 * c) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < R; ++u) {
                dot[u] += qv.x * x[u].x + qv.y * x[u].y + qv.z * x[u].z + qv.w * x[u].w;
                sq[u] += x[u].x * x[u].x + x[u].y * x[u].y + x[u].z * x[u].z + x[u].w * x[u].w;
            }
        }
#pragma unroll
        for (int u = 0; u < R; ++u) {
            const int r = r0 + u;
            const float dt = iq_warp_sum(dot[u]);
            const float s2 = normalize_rows ? iq_warp_sum(sq[u]) : 0.f;
            if (r < n) {
                const float sim = normalize_rows ? dt * qinv * (1.f / sqrtf(s2 + 1e-8f)) : dt * qinv;
                if (sims && lane == 0) sims[r] = sim;
                if (k > 0) iq_insert(val, idx, k, sim, r, lane);
            }
        }
    }
    if (k <= 0) return;
    if (lane < k) { s_val[warp][lane] = val; s_idx[warp][lane] = idx; }
    __syncthreads();
    if (warp == 0) {
        for (int w = 1; w < kIqWarps; ++w)
            for (int s = 0; s < k; ++s) {
                const float v = s_val[w][s];
                const int iv = s_idx[w][s];
                if (iv != INT_MAX) iq_insert(val, idx, k, v, iv, lane);
            }
        if (lane < k) {
            cand_val[(size_t)blockIdx.x * k + lane] = val;
            cand_idx[(size_t)blockIdx.x * k + lane] = idx;
        }
    }
}

// Pass 2: merge ncand candidate lists of k (one CTA of 32 warps).
__global__ void __launch_bounds__(kIqMergeThreads) index_merge_kernel(const float* __restrict__ cand_val,
                                                                      const int* __restrict__ cand_idx, int nlists,
                                                                      int k, float* __restrict__ top_val,
                                                                      int32_t* __restrict__ top_idx) {
    constexpr int W = kIqMergeThreads / 32;
    __shared__ float s_val[W][kIqMaxK];
    __shared__ int s_idx[W][kIqMaxK];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float val = -FLT_MAX;
    int idx = INT_MAX;
    const int total = nlists * k;
    for (int base = warp * 32; base < total; base += W * 32) {
        const int e = base + lane;
        const float v = e < total ? cand_val[e] : -FLT_MAX;
        const int iv = e < total ? cand_idx[e] : INT_MAX;
        for (int j = 0; j < 32; ++j) {
            const float vj = __shfl_sync(0xffffffffu, v, j);
            const int ij = __shfl_sync(0xffffffffu, iv, j);
            if (ij != INT_MAX) iq_insert(val, idx, k, vj, ij, lane);
        }
    }
    if (lane < k) { s_val[warp][lane] = val; s_idx[warp][lane] = idx; }
    __syncthreads();
    if (warp == 0) {
        for (int w = 1; w < W; ++w)
            for (int s = 0; s < k; ++s)
                if (s_idx[w][s] != INT_MAX) iq_insert(val, idx, k, s_val[w][s], s_idx[w][s], lane);
        if (lane < k) {
            top_val[lane] = idx == INT_MAX ? -FLT_MAX : val;
            top_idx[lane] = idx == INT_MAX ? -1 : idx;
        }
    }
}

int iq_grid(int n) {
    const int per_cta = kIqWarps * 4;                      // rows per CTA per grid-stride step
    int g = (n + per_cta - 1) / per_cta;
    const int cap = sm_count() * 8;                        // 8 CTAs of 8 warps per SM
    return g < 1 ? 1 : (g > cap ? cap : g);
}

}  // namespace
}  // namespace kessie

using namespace kessie;

extern "C" size_t kessie_index_query_workspace_size(int num_rows, int top_k) {
    if (num_rows <= 0 || top_k <= 0 || top_k > kIqMaxK) return 0;
    return (size_t)iq_grid(num_rows) * top_k * (sizeof(float) + sizeof(int)) + 256;
}

extern "C" int kessie_index_query_v2(const float* query, const float* index, int num_rows, int dim,
                                     int normalize_rows, float* sims, int top_k, int32_t* top_idx, float* top_scores,
                                     void* workspace, size_t workspace_bytes, void* stream) {
    if (!query || !index || num_rows <= 0 || dim <= 0 || dim % 4 || top_k < 0 || top_k > kIqMaxK)
        return set_error(KESSIE_ERR_ARG, "index_query_v2: bad arguments (dim %% 4 == 0, 0 <= top_k <= %d)", kIqMaxK);
    if ((reinterpret_cast<uintptr_t>(query) | reinterpret_cast<uintptr_t>(index)) & 15)
        return set_error(KESSIE_ERR_ARG, "index_query_v2: query / index must be 16-byte aligned");
    if (top_k > 0 && (!top_idx || !top_scores))
        return set_error(KESSIE_ERR_ARG, "index_query_v2: top_k > 0 needs top_idx and top_scores");
    if (top_k == 0 && !sims) return set_error(KESSIE_ERR_ARG, "index_query_v2: nothing to output");
    const int grid = iq_grid(num_rows);
    float* cv = nullptr;
    int* ci = nullptr;
    if (top_k > 0) {
        const size_t need = kessie_index_query_workspace_size(num_rows, top_k);
        if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 15))
            return set_error(KESSIE_ERR_WORKSPACE, "index_query_v2: workspace %zu < %zu", workspace_bytes, need);
        cv = static_cast<float*>(workspace);
        ci = reinterpret_cast<int*>(cv + (size_t)grid * top_k);
    }
    cudaStream_t st = as_stream(stream);
    index_query_kernel<<<grid, kIqThreads, 0, st>>>(query, index, num_rows, dim, normalize_rows ? 1 : 0, sims, top_k,
                                                    cv, ci);
    int rc = check_launch("index_query");
    if (rc || top_k == 0) return rc;
    index_merge_kernel<<<1, kIqMergeThreads, 0, st>>>(cv, ci, grid, top_k, top_scores, top_idx);
    return check_launch("index_query merge");
}
