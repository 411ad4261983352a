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
// Design (B200, HBM-bound: N * dim * 4 bytes per query): eight lanes per
// row, so one warp covers four rows per step and each lane has eight 16-byte
// chunks of its row in flight at once (a whole 256-float row slice in one
// load round); a three-step shuffle gives the row's dot product and squared
// norm.  Every warp keeps its running top-k in registers (lane s holds rank s,
// lanes >= k hold worse entries or sentinels) with the k-th entry as a
// threshold: a ballot offers the four rows at once and only rows above the
// threshold are inserted (ballot + shuffle-up), so once the list fills a step
// costs one ballot.  Lists are combined with bitonic networks across the 32
// lanes (sort 32 / merge two sorted 32-lists: five shuffle stages each): the
// CTA folds its warps' lists as a tree and writes one list; a one-CTA second
// launch takes the k best list heads, and only the k lists they head can hold
// the global top-k, so at most k * k candidates go through the final tree.
#include "common.cuh"
#include "ptx.cuh"

#include <float.h>

namespace kessie {
namespace {

constexpr int kIqWarps = 8;
constexpr int kIqThreads = kIqWarps * 32;
constexpr int kIqMaxK = 32;
constexpr int kIqMergeThreads = 1024;
constexpr int kIqLanesPerRow = 8;
constexpr int kIqRowsPerStep = 32 / kIqLanesPerRow;        // rows per warp step
constexpr int kIqUnroll = 8;                               // 16-byte chunks in flight per lane
constexpr int kIqMinBlocks = 4;                            // resident CTAs per SM
constexpr unsigned kFull = 0xffffffffu;

// (score, index) order: higher score first, lower index first on ties.  A
// strict total order, so the selected set and its order do not depend on the
// order in which rows are offered; (-FLT_MAX, INT_MAX) is the empty sentinel.
__device__ __forceinline__ bool iq_better(float a, int ia, float b, int ib) {
    return a > b || (a == b && ia < ib);
}

// Compare-exchange with lane ^ m: keep the better entry when keep_better.
__device__ __forceinline__ void iq_cas(float& v, int& i, int m, bool keep_better) {
    const float ov = __shfl_xor_sync(kFull, v, m);
    const int oi = __shfl_xor_sync(kFull, i, m);
    if (iq_better(ov, oi, v, i) == keep_better) { v = ov; i = oi; }
}

// Bitonic sort of one entry per lane, best first.
__device__ __forceinline__ void iq_sort32(float& v, int& i, int lane) {
#pragma unroll
    for (int size = 2; size <= 32; size <<= 1)
#pragma unroll
        for (int m = size >> 1; m > 0; m >>= 1)
            iq_cas(v, i, m, ((lane & m) == 0) == ((lane & size) == 0));
}

// (v, i) <- best 32 of two lists sorted best first, sorted best first.
__device__ __forceinline__ void iq_merge32(float& v, int& i, float bv, int bi, int lane) {
    const float rv = __shfl_sync(kFull, bv, 31 - lane);
    const int ri = __shfl_sync(kFull, bi, 31 - lane);
    if (iq_better(rv, ri, v, i)) { v = rv; i = ri; }      // bitonic: the best 32 of both
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) iq_cas(v, i, m, (lane & m) == 0);
}

// Tree fold of the sorted lists of warps [0, nact) into warp 0 (block-wide
// call: every thread reaches the barriers; nact is block-uniform).
__device__ __forceinline__ void iq_block_fold(float& v, int& i, float* s_v, int* s_i, int nact, int warp,
                                              int lane) {
    int span = 1;
    while (span < nact) span <<= 1;
    if (warp < nact) { s_v[warp * 32 + lane] = v; s_i[warp * 32 + lane] = i; }
    for (int half = span >> 1; half >= 1; half >>= 1) {
        __syncthreads();
        if (warp < half && warp + half < nact) {
            iq_merge32(v, i, s_v[(warp + half) * 32 + lane], s_i[(warp + half) * 32 + lane], lane);
            s_v[warp * 32 + lane] = v;
            s_i[warp * 32 + lane] = i;
        }
    }
}

// A warp's top-k list: lane s < k holds rank s; (tv, ti) is the k-th entry.
struct IqList {
    float val = -FLT_MAX, tv = -FLT_MAX;
    int idx = INT_MAX, ti = INT_MAX;

    // Offer one (v, iv) per lane where ok is set (warp-wide call).
    __device__ __forceinline__ void offer(int k, float v, int iv, bool ok, int lane) {
        unsigned m = __ballot_sync(kFull, ok && iq_better(v, iv, tv, ti));
        while (m) {
            const int src = __ffs(m) - 1;
            m &= m - 1;
            const float cv = __shfl_sync(kFull, v, src);
            const int ci = __shfl_sync(kFull, iv, src);
            if (!iq_better(cv, ci, tv, ti)) continue;      // warp-uniform
            const int pos = __popc(__ballot_sync(kFull, lane < k && iq_better(val, idx, cv, ci)));
            const float up_v = __shfl_up_sync(kFull, val, 1);
            const int up_i = __shfl_up_sync(kFull, idx, 1);
            if (lane < k) {
                if (lane > pos) { val = up_v; idx = up_i; }
                else if (lane == pos) { val = cv; idx = ci; }
            }
            tv = __shfl_sync(kFull, val, k - 1);
            ti = __shfl_sync(kFull, idx, k - 1);
        }
    }
};

// Pass 1: similarities (optional output) and one top-k list per CTA.
template <bool NORM>
__global__ void __launch_bounds__(kIqThreads, kIqMinBlocks) index_query_kernel(
    const float* __restrict__ query, const float* __restrict__ index, int n, int dim, float* __restrict__ sims, int k,
    float* __restrict__ cand_val, int* __restrict__ cand_idx) {
    __shared__ float s_val[kIqWarps * 32];
    __shared__ int s_idx[kIqWarps * 32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // the merge launch (programmatic dependent launch) may be scheduled now:
    // it waits for this grid's completion before reading the lists
    ptx::launch_dependents();
    const int d4 = dim >> 2;                               // 16-byte chunks per row
    const float4* q4 = reinterpret_cast<const float4*>(query);
    float qq = 0.f;
    for (int c = lane; c < d4; c += 32) {
        const float4 x = __ldg(q4 + c);
        qq += x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) qq += __shfl_xor_sync(kFull, qq, o);
    const float qinv = 1.f / sqrtf(qq + 1e-8f);
    const int sub = lane % kIqLanesPerRow, rsub = lane / kIqLanesPerRow;
    IqList list;
    const int gw = blockIdx.x * kIqWarps + warp, nw = gridDim.x * kIqWarps;
    const int wstride = nw * kIqRowsPerStep;
    for (long long r0 = (long long)gw * kIqRowsPerStep; r0 < n; r0 += wstride) {
        const int r = (int)min(r0 + rsub, (long long)INT_MAX);
        const bool live = r < n;
        const float4* x4 = reinterpret_cast<const float4*>(index + (size_t)(live ? r : 0) * dim);
        float dot = 0.f, sq = 0.f;
        for (int c0 = sub; c0 < d4; c0 += kIqLanesPerRow * kIqUnroll) {
            float4 x[kIqUnroll];
#pragma unroll
            for (int u = 0; u < kIqUnroll; ++u) {
                const int c = c0 + u * kIqLanesPerRow;
                x[u] = (live && c < d4) ? ldg_stream_f4(reinterpret_cast<const float*>(x4 + c))
                                        : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < kIqUnroll; ++u) {
                const int c = c0 + u * kIqLanesPerRow;
                const float4 qv = c < d4 ? __ldg(q4 + c) : make_float4(0.f, 0.f, 0.f, 0.f);
                dot += qv.x * x[u].x + qv.y * x[u].y + qv.z * x[u].z + qv.w * x[u].w;
                if (NORM) sq += x[u].x * x[u].x + x[u].y * x[u].y + x[u].z * x[u].z + x[u].w * x[u].w;
            }
        }
#pragma unroll
        for (int o = 1; o < kIqLanesPerRow; o <<= 1) {
            dot += __shfl_xor_sync(kFull, dot, o);
            if (NORM) sq += __shfl_xor_sync(kFull, sq, o);
        }
        const float sim = NORM ? dot * qinv * (1.f / sqrtf(sq + 1e-8f)) : dot * qinv;
        const bool lead = live && sub == 0;
        if (sims && lead) sims[r] = sim;
        if (k > 0) list.offer(k, sim, r, lead, lane);
    }
    if (k <= 0) return;                                    // block-uniform
    float v = list.val;
    int i = list.idx;
    iq_block_fold(v, i, s_val, s_idx, kIqWarps, warp, lane);
    if (warp == 0 && lane < k) {
        cand_val[(size_t)blockIdx.x * k + lane] = v;
        cand_idx[(size_t)blockIdx.x * k + lane] = i;
    }
}

// Pass 2: merge nlists sorted candidate lists of k (one CTA of 32 warps).
__global__ void __launch_bounds__(kIqMergeThreads) index_merge_kernel(const float* __restrict__ cand_val,
                                                                      const int* __restrict__ cand_idx, int nlists,
                                                                      int k, float* __restrict__ top_val,
                                                                      int32_t* __restrict__ top_idx) {
    constexpr int W = kIqMergeThreads / 32;
    __shared__ float s_val[W * 32];
    __shared__ int s_idx[W * 32];
    __shared__ int s_sel[32];
    __shared__ int s_nsel;
    __shared__ float s_tv;
    __shared__ int s_ti;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    ptx::grid_dependency_wait();                           // pass 1 complete, its lists visible
    if (threadIdx.x == 0) s_nsel = 0;
    // 1. the k best list heads (each list is sorted, best first)
    float v = -FLT_MAX;
    int i = INT_MAX;
    for (int b = warp * 32; b < nlists; b += kIqMergeThreads) {
        const int l = b + lane;
        float hv = -FLT_MAX;
        int hi = INT_MAX;
        if (l < nlists) { hv = cand_val[(size_t)l * k]; hi = cand_idx[(size_t)l * k]; }
        iq_sort32(hv, hi, lane);
        iq_merge32(v, i, hv, hi, lane);
    }
    const int nact = min(W, (nlists + 31) / 32);
    iq_block_fold(v, i, s_val, s_idx, nact, warp, lane);
    if (warp == 0) {
        const float tv = __shfl_sync(kFull, v, k - 1);
        const int ti = __shfl_sync(kFull, i, k - 1);
        if (lane == 0) { s_tv = tv; s_ti = ti; }
    }
    __syncthreads();
    // 2. the lists headed by those k heads hold every entry of the top-k
    const float tv = s_tv;
    const int ti = s_ti;
    for (int l = threadIdx.x; l < nlists; l += kIqMergeThreads) {
        const float hv = cand_val[(size_t)l * k];
        const int hi = cand_idx[(size_t)l * k];
        if (hi != INT_MAX && !iq_better(tv, ti, hv, hi)) {
            const int slot = atomicAdd(&s_nsel, 1);
            if (slot < 32) s_sel[slot] = l;
        }
    }
    __syncthreads();
    const int nsel = min(s_nsel, 32);
    const int ncand = nsel * k;
    v = -FLT_MAX;
    i = INT_MAX;
    if ((int)threadIdx.x < ncand) {
        const size_t e = (size_t)s_sel[threadIdx.x / k] * k + threadIdx.x % k;
        v = cand_val[e];
        i = cand_idx[e];
    }
    const int nact2 = max(1, (ncand + 31) / 32);
    if (warp < nact2) iq_sort32(v, i, lane);
    iq_block_fold(v, i, s_val, s_idx, nact2, warp, lane);
    if (warp == 0 && lane < k) {
        top_val[lane] = i == INT_MAX ? -FLT_MAX : v;
        top_idx[lane] = i == INT_MAX ? -1 : i;
    }
}

// One wave of resident CTAs at most, sized so that every warp gets the same
// number of row steps (the last DRAM round then has every warp loading).
int iq_grid(int n) {
    const long long steps = ((long long)n + kIqRowsPerStep - 1) / kIqRowsPerStep;
    const long long max_warps = (long long)sm_count() * kIqMinBlocks * kIqWarps;
    const long long per_warp = (steps + max_warps - 1) / max_warps;
    const long long warps = (steps + per_warp - 1) / per_warp;
    const long long g = (warps + kIqWarps - 1) / kIqWarps;
    return (int)(g < 1 ? 1 : g);
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
    NvtxRange nvtx_range("kessie_index_query_v2");
    if (!query || !index || num_rows <= 0 || dim <= 0 || dim % 4 || dim > (1 << 24) || top_k < 0 || top_k > kIqMaxK)
        return set_error(KESSIE_ERR_ARG, "index_query_v2: bad arguments (0 < dim <= 2^24, dim %% 4 == 0, 0 <= top_k <= %d)", kIqMaxK);
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
    if (normalize_rows)
        index_query_kernel<true><<<grid, kIqThreads, 0, st>>>(query, index, num_rows, dim, sims, top_k, cv, ci);
    else
        index_query_kernel<false><<<grid, kIqThreads, 0, st>>>(query, index, num_rows, dim, sims, top_k, cv, ci);
    int rc = check_launch("index_query");
    if (rc || top_k == 0) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(kIqMergeThreads);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, index_merge_kernel, (const float*)cv, (const int*)ci, grid, top_k,
                                             top_scores, top_idx);
    if (e != cudaSuccess) return set_error(KESSIE_ERR_CUDA, "index_query merge: %s", cudaGetErrorString(e));
    return check_launch("index_query merge");
}
