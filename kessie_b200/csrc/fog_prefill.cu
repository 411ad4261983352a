// fog_prefill.cu -- fog attention over many query rows (chunked prefill, and
// the legacy dense [B,H,N,D] windowed / fused-fog launchers).
//
// Semantics: kessie_windowed_attention_ref / kessie_fused_fog_attention_ref
// (kessie_hip_kernels.py:577-593) with a query offset (query i sits at
// absolute position q_start + i), GQA, and a paged or dense KV:
//   mask  causal: j <= i_abs;  window W > 0: 0 <= i_abs - j < W
//   O_i = sum_j p_ij w_j v_j / sum_j p_ij   (fog scales V only)
//
// Layout and pipeline (shared with the decode kernel): K/V arrive as
// 16-token TMA boxes ([D/64][16][64] elements, 128-byte swizzle) addressed
// through a 5-D tensor map [64][token][D/64][head][page].  The dense layout
// [B,H,N,D] is the same map with page = batch and token = position (boxes past
// N are zero-filled by TMA).  A CTA owns 64 query rows of one KV head (rows
// are (token, head-in-group) pairs, so the Hq/Hkv query heads that share a
// KV head share every K/V tile), a producer warp streams 64-key tiles through
// a 3-stage mbarrier ring, and 4 consumer warps (16 rows each) run the
// warp-level tensor-core flash-attention recurrence:
//   S = Q K^T (mma.sync m16n8k16), mask, online softmax (quad shuffles),
//   P' = P * w_j, O += P' V (ldmatrix.trans of V).
#include "common.cuh"
#include "decode_f32.cuh"
#include "ptx.cuh"
#include "tma_host.cuh"
#include "prefill_common.cuh"

#include <math.h>

#include <algorithm>

namespace kessie {
namespace {

constexpr int kPW = 4;            // consumer warps (16 rows each)
constexpr int kBM = 16 * kPW;     // query rows per CTA
constexpr int kBN = 64;           // keys per tile
constexpr int kPST = 3;           // stages
constexpr int kPThreads = (kPW + 1) * 32;
constexpr float kLog2e = 1.4426950408889634f;



template <int D>
struct PSmem {
    static constexpr int kBox = 16 * D * 2;          // one 16-token box
    static constexpr int kTile = 4 * kBox;           // 64 keys
    static constexpr int kStage = 2 * kTile;         // K + V
    static constexpr int kBarOff = kPST * kStage;
    static constexpr int kAlloc = kBarOff + 2 * kPST * 8 + 1024;
};

__device__ __forceinline__ uint32_t swz(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

// Offset of (key k in a 64-key tile, 16B chunk ch of the row) in a tile.
template <int D>
__device__ __forceinline__ uint32_t tile_off(int k, int ch) {
    return (uint32_t)((k >> 4) * PSmem<D>::kBox) + swz((ch >> 3) * 16 + (k & 15), ch & 7);
}

__device__ __forceinline__ float fogw(const PrefillParams& p, int b, int cs, int j) {
    if (p.fog_w) return __ldg(p.fog_w + b * p.fog_w_sb + j);
    if (j >= cs) return 1.f;
    return powf(__fdiv_rn((float)j, (float)max(cs - 1, 1)), p.fog_alpha);
}

template <int D, bool BF16>
__global__ void __launch_bounds__(kPThreads, 1) fog_prefill_kernel(const __grid_constant__ CUtensorMap tmK,
                                                                    const __grid_constant__ CUtensorMap tmV,
                                                                    const PrefillParams p) {
    using S = PSmem<D>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kBarOff);
    uint64_t* empty = full + kPST;

    // heavy (late, causal) row tiles first
    const int tile_m = gridDim.x - 1 - blockIdx.x;
    const int hk = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rows_total = p.Nq * p.G;
    const int row0 = tile_m * kBM;
    const int kv_len = p.kv_lens ? p.kv_lens[b] : p.kv_len_const;
    // query 0 position: explicit, constant, or (q_start_const < 0) the last Nq keys
    const int q0 = p.q_start ? p.q_start[b] : (p.q_start_const >= 0 ? p.q_start_const : kv_len - p.Nq);
    // absolute positions of the CTA's first / last query token
    const int t_first = row0 / p.G;
    const int t_last = min(row0 + kBM, rows_total) - 1;
    const int pos_lo = q0 + t_first, pos_hi = q0 + t_last / p.G;
    int j_lo = p.window > 0 ? max(0, pos_lo - p.window + 1) : 0;
    int j_hi = (p.causal || p.window > 0) ? min(kv_len, pos_hi + 1) : kv_len;
    if (j_hi < j_lo) j_hi = j_lo;
    const int tile_lo = j_lo / kBN, tile_hi = (j_hi + kBN - 1) / kBN;
    const int n_tiles = tile_hi - tile_lo;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kPST; ++s) { ptx::mbar_init(&full[s], 1); ptx::mbar_init(&empty[s], kPW); }
        ptx::fence_mbar_init();
    }
    __syncthreads();

    // ------------------------------------------------------------ producer warp
    if (warp == kPW) {
        const int32_t* bt = p.block_table ? p.block_table + (int64_t)b * p.bt_stride : nullptr;
        const int kv_pages = p.block_table ? (kv_len + 16 * p.upp - 1) / (16 * p.upp) : 0;
        uint64_t pol = ptx::policy_evict_first();
        int ids_reg = 0, ids_base = -1000000;
        int issued = 0;
        for (int it = 0; it < n_tiles; ++it) {
            const int tile = tile_lo + it;
            // page ids for this tile's 4 boxes: one warp-wide load covers 8 tiles
            int page[4];
            if (bt) {
                const int unit0 = tile * 4;               // 16-token units
                if ((unit0 + 3) / p.upp >= ids_base + 32 || unit0 / p.upp < ids_base) {
                    ids_base = unit0 / p.upp;
                    const int pi = ids_base + lane;
                    int id = pi < kv_pages ? __ldg(bt + pi) : -1;
                    if (pi < kv_pages && (id < 0 || id >= p.num_pages)) { record_status(p.status, KESSIE_DEV_BAD_PAGE_ID); id = -1; }
                    ids_reg = id;
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int pi = (unit0 + u) / p.upp;
                    int id = __shfl_sync(0xffffffffu, ids_reg, (pi - ids_base) & 31);
                    if (pi - ids_base >= 32) id = -1;     // cannot happen: 4 units span at most 4 pages
                    page[u] = id;
                }
            }
            if (lane == 0) {
                const int s = it % kPST;
                if (it >= kPST && !ptx::mbar_wait(&empty[s], ((uint32_t)(it / kPST) & 1u) ^ 1u)) {
                    record_status(p.status, KESSIE_DEV_WAIT_TIMEOUT);
                    issued = -issued - 1;
                } else {
                    ptx::mbar_arrive_expect_tx(&full[s], (uint32_t)S::kStage);
                    uint8_t* st = smem + s * S::kStage;
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        int c1, c4;
                        if (bt) {
                            const int unit = tile * 4 + u;
                            c1 = (unit % p.upp) * 16;
                            c4 = page[u] < 0 ? p.num_pages : page[u];
                        } else {
                            c1 = tile * kBN + u * 16;
                            c4 = b;
                        }
                        ptx::tma_load_5d_hint(st + u * S::kBox, &tmK, &full[s], 0, c1, 0, hk, c4, pol);
                        ptx::tma_load_5d_hint(st + S::kTile + u * S::kBox, &tmV, &full[s], 0, c1, 0, hk, c4, pol);
                    }
                    issued = it + 1;
                }
            }
            issued = __shfl_sync(0xffffffffu, issued, 0);
            if (issued < 0) { issued = -issued - 1; break; }
        }
        if (lane == 0) {
            for (int it = max(0, issued - kPST); it < issued; ++it)
                if (!ptx::mbar_wait(&full[it % kPST], (uint32_t)(it / kPST) & 1u)) {
                    record_status(p.status, KESSIE_DEV_WAIT_TIMEOUT);
                    break;
                }
        }
        return;
    }

    // ------------------------------------------------------------ consumers
    const int g = lane >> 2, t = lane & 3;
    const int rA = row0 + warp * 16 + g, rB = rA + 8;         // this thread's two rows
    const bool okA = rA < rows_total, okB = rB < rows_total;
    const int tokA = rA / p.G, tokB = rB / p.G;
    const int posA = q0 + tokA, posB = q0 + tokB;
    // Q A-fragments: a0 = Q[rA][kk*16+2t..], a1 = Q[rB][..], a2 = Q[rA][+8], a3 = Q[rB][+8]
    uint32_t qa[D / 16][4];
    {
        const uint16_t* base = reinterpret_cast<const uint16_t*>(p.q) + (int64_t)b * p.q_sb;
        const uint16_t* qA = base + (int64_t)(okA ? tokA : 0) * p.q_st + (int64_t)(hk * p.G + (okA ? rA % p.G : 0)) * p.q_sh;
        const uint16_t* qB = base + (int64_t)(okB ? tokB : 0) * p.q_st + (int64_t)(hk * p.G + (okB ? rB % p.G : 0)) * p.q_sh;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
            qa[kk][0] = okA ? *reinterpret_cast<const uint32_t*>(qA + kk * 16 + 2 * t) : 0u;
            qa[kk][1] = okB ? *reinterpret_cast<const uint32_t*>(qB + kk * 16 + 2 * t) : 0u;
            qa[kk][2] = okA ? *reinterpret_cast<const uint32_t*>(qA + kk * 16 + 2 * t + 8) : 0u;
            qa[kk][3] = okB ? *reinterpret_cast<const uint32_t*>(qB + kk * 16 + 2 * t + 8) : 0u;
        }
    }
    float o[D / 8][4];
#pragma unroll
    for (int n = 0; n < D / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;
    const int cs = (p.clear_start || p.clear_start_const > 0) && p.fog_alpha > 0.f
                       ? (p.clear_start ? p.clear_start[b] : p.clear_start_const) : INT_MIN;
    const bool has_fog = p.fog_w != nullptr || cs > 0;
    const bool has_bias = p.bias.on != 0;
    const int bias_fb = has_bias ? fog_bias_boundary(p.bias, kv_len) : 0;

    const int mi = lane >> 3, rr = lane & 7;
    const int kkey = rr + 8 * (mi >> 1), kch = mi & 1;     // K (B operand, non-trans)
    const int vkey = rr + 8 * (mi & 1), vch = mi >> 1;     // V (B operand, trans)

    for (int it = 0; it < n_tiles; ++it) {
        const int s = it % kPST;
        // warp-uniform: the ldmatrix / mma.sync below are warp-collective
        if (!__all_sync(0xffffffffu, ptx::mbar_wait(&full[s], (uint32_t)(it / kPST) & 1u))) {
            if (lane == 0) record_status(p.status, KESSIE_DEV_WAIT_TIMEOUT);
            break;
        }
        const int j0 = (tile_lo + it) * kBN;
        uint8_t* kt = smem + s * S::kStage;
        uint8_t* vt = kt + S::kTile;
        // paged caches: zero V rows past kv_len (stale slots of the last page)
        if (p.block_table && j0 + kBN > kv_len) {
            for (int e = lane; e < kBN * (D / 8); e += 32) {
                const int key = e % kBN, ch = e / kBN;
                if (j0 + key >= kv_len) *reinterpret_cast<uint4*>(vt + tile_off<D>(key, ch)) = make_uint4(0, 0, 0, 0);
            }
            __syncwarp();
        }
        // ---- S = Q K^T  (16 rows x 64 keys)
        float sc[8][4];
#pragma unroll
        for (int n = 0; n < 8; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
        const uint32_t kb = ptx::smem_u32(kt);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
            for (int np = 0; np < 4; ++np) {
                uint32_t b0, b1, b2, b3;
                ptx::ldmatrix_x4(b0, b1, b2, b3, kb + tile_off<D>(np * 16 + kkey, kk * 2 + kch));
                ptx::mma_16816<BF16>(sc[2 * np], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b0, b1);
                ptx::mma_16816<BF16>(sc[2 * np + 1], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b2, b3);
            }
        }
        // ---- mask + online softmax (rows A: c0,c1; rows B: c2,c3)
        float mxA = -INFINITY, mxB = -INFINITY;
#pragma unroll
        for (int n = 0; n < 8; ++n) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int j = j0 + n * 8 + 2 * t + e;
                bool vA = j < kv_len && okA, vB = j < kv_len && okB;
                if (p.causal) { vA = vA && j <= posA; vB = vB && j <= posB; }
                if (p.window > 0) {
                    vA = vA && j <= posA && posA - j < p.window;
                    vB = vB && j <= posB && posB - j < p.window;
                }
                const float bj = (has_bias && j < kv_len) ? fog_bias_at(p.bias, bias_fb, j) * kLog2e : 0.f;
                sc[n][e] = vA ? fmaf(sc[n][e], p.scale_log2, bj) : -INFINITY;
                sc[n][2 + e] = vB ? fmaf(sc[n][2 + e], p.scale_log2, bj) : -INFINITY;
                mxA = fmaxf(mxA, sc[n][e]);
                mxB = fmaxf(mxB, sc[n][2 + e]);
            }
        }
        mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, 1));
        mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, 2));
        mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, 1));
        mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, 2));
        const float mnA = fmaxf(mA, mxA), mnB = fmaxf(mB, mxB);
        const float bA = mnA == -INFINITY ? 0.f : mnA, bB = mnB == -INFINITY ? 0.f : mnB;
        const float alA = exp2f(mA - bA), alB = exp2f(mB - bB);
        mA = mnA; mB = mnB;
        float sumA = 0.f, sumB = 0.f;
        uint32_t pa[4][4];      // A fragments of P' for 4 k-steps of 16 keys
#pragma unroll
        for (int n = 0; n < 8; ++n) {
            const float p0 = exp2f(sc[n][0] - bA), p1 = exp2f(sc[n][1] - bA);
            const float p2 = exp2f(sc[n][2] - bB), p3 = exp2f(sc[n][3] - bB);
            sumA += p0 + p1; sumB += p2 + p3;
            float w0 = 1.f, w1 = 1.f;
            if (has_fog) {
                const int j = j0 + n * 8 + 2 * t;
                w0 = j < kv_len ? fogw(p, b, cs, j) : 0.f;
                w1 = j + 1 < kv_len ? fogw(p, b, cs, j + 1) : 0.f;
            }
            const int ks = n >> 1, hi = n & 1;
            pa[ks][hi * 2 + 0] = ptx::pack2<BF16>(p0 * w0, p1 * w1);
            pa[ks][hi * 2 + 1] = ptx::pack2<BF16>(p2 * w0, p3 * w1);
        }
        lA = lA * alA + sumA;
        lB = lB * alB + sumB;
#pragma unroll
        for (int n = 0; n < D / 8; ++n) { o[n][0] *= alA; o[n][1] *= alA; o[n][2] *= alB; o[n][3] *= alB; }
        // ---- O += P' V
        const uint32_t vb = ptx::smem_u32(vt);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
            for (int dp = 0; dp < D / 16; ++dp) {
                uint32_t b0, b1, b2, b3;
                ptx::ldmatrix_x4_trans(b0, b1, b2, b3, vb + tile_off<D>(ks * 16 + vkey, dp * 2 + vch));
                // a-frag order: a0 = rows A keys lo, a1 = rows B keys lo, a2 = rows A keys hi, a3 = rows B keys hi
                ptx::mma_16816<BF16>(o[2 * dp], pa[ks][0], pa[ks][1], pa[ks][2], pa[ks][3], b0, b1);
                ptx::mma_16816<BF16>(o[2 * dp + 1], pa[ks][0], pa[ks][1], pa[ks][2], pa[ks][3], b2, b3);
            }
        }
        if (p.block_table && j0 + kBN > kv_len) ptx::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&empty[s]);
    }
    // ---- epilogue
    lA += __shfl_xor_sync(0xffffffffu, lA, 1); lA += __shfl_xor_sync(0xffffffffu, lA, 2);
    lB += __shfl_xor_sync(0xffffffffu, lB, 1); lB += __shfl_xor_sync(0xffffffffu, lB, 2);
    const float iA = lA > 0.f ? 1.f / lA : 0.f, iB = lB > 0.f ? 1.f / lB : 0.f;
    uint16_t* ob = reinterpret_cast<uint16_t*>(p.o) + (int64_t)b * p.o_sb;
    if (okA) {
        uint16_t* orow = ob + (int64_t)tokA * p.o_st + (int64_t)(hk * p.G + rA % p.G) * p.o_sh;
#pragma unroll
        for (int n = 0; n < D / 8; ++n)
            *reinterpret_cast<uint32_t*>(orow + n * 8 + 2 * t) = ptx::pack2<BF16>(o[n][0] * iA, o[n][1] * iA);
    }
    if (okB) {
        uint16_t* orow = ob + (int64_t)tokB * p.o_st + (int64_t)(hk * p.G + rB % p.G) * p.o_sh;
#pragma unroll
        for (int n = 0; n < D / 8; ++n)
            *reinterpret_cast<uint32_t*>(orow + n * 8 + 2 * t) = ptx::pack2<BF16>(o[n][2] * iB, o[n][3] * iB);
    }
}

template <int D, bool BF16>
int launch_prefill_t(const CUtensorMap& mk, const CUtensorMap& mv, const PrefillParams& p, cudaStream_t st) {
    auto kern = fog_prefill_kernel<D, BF16>;
    const int smem = PSmem<D>::kAlloc;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
        return check_launch("prefill: set smem attribute");
    const int rows = p.Nq * p.G;
    dim3 grid((rows + kBM - 1) / kBM, p.Hkv, p.B);
    kern<<<grid, kPThreads, smem, st>>>(mk, mv, p);
    return check_launch("fog_prefill");
}

int run_prefill(const PrefillParams& p, const void* kc, const void* vc, int64_t page_stride, int64_t token_stride,
                int64_t head_stride, int map_pages, int map_tokens, int D, bool bf16, cudaStream_t st) {
    // tcgen05/TMEM kernel for the shapes it covers (head_dim 128, Hq/Hkv | 128)
    const int rc = run_prefill_tc(p, p.q, kc, vc, page_stride, token_stride, head_stride, map_pages, map_tokens, D,
                                  bf16, st);
    if (rc != kTcNotCovered) return rc;
    CUtensorMap mk, mv;
    CUresult r1 = encode_kv_tile_map(&mk, kc, bf16, D, map_tokens, p.Hkv, map_pages, token_stride, head_stride, page_stride);
    CUresult r2 = encode_kv_tile_map(&mv, vc, bf16, D, map_tokens, p.Hkv, map_pages, token_stride, head_stride, page_stride);
    if (r1 != CUDA_SUCCESS || r2 != CUDA_SUCCESS)
        return set_error(KESSIE_ERR_ARG, "prefill: TMA descriptor rejected (%d/%d)", (int)r1, (int)r2);
    if (D == 128) return bf16 ? launch_prefill_t<128, true>(mk, mv, p, st) : launch_prefill_t<128, false>(mk, mv, p, st);
    return bf16 ? launch_prefill_t<64, true>(mk, mv, p, st) : launch_prefill_t<64, false>(mk, mv, p, st);
}

// Copy the first kv_len keys of every sequence from the paged cache into a
// head-major staging buffer [B][Hkv][kv_max][D] (K and V), zero-filling rows
// [kv_len, kv_pad) so the tile that straddles kv_len reads zeros.  The
// tcgen05 prefill then streams 128-token TMA boxes from contiguous memory
// instead of 16-token boxes scattered over pages (a TMA box costs a fixed
// ~130 SM cycles, so 2 KB boxes cannot feed the tensor cores).
// The fog weight of each key (kessie_hip_kernels.py:408-412: the fp32 ratio
// j / max(cs-1, 1), then pow) is folded into the staged V here, once per key:
// O = sum_j p_j (w_j v_j) / sum_j p_j is the same sum, and the attention
// kernels then run without per-key weights on their softmax path.
// grid (ceil(kv_max / page_size), B); threads over (kv, head, 16-byte chunk).
template <typename T>
__global__ void __launch_bounds__(256) stage_kv_kernel(const T* __restrict__ kc, const T* __restrict__ vc,
                                                       int64_t page_stride, int64_t token_stride, int64_t head_stride,
                                                       int num_pages, int ps, const int32_t* __restrict__ bt,
                                                       int64_t bt_stride, const int32_t* __restrict__ kv_lens,
                                                       int max_kv_len, int kv_max, int Hkv, int D,
                                                       const int32_t* __restrict__ clear_start, float fog_alpha,
                                                       const float* __restrict__ fog_w, int64_t fog_w_sb,
                                                       T* __restrict__ sk, T* __restrict__ sv, int* status) {
    __shared__ float wts[256];
    const int pg = blockIdx.x, b = blockIdx.y;
    int kv_len = kv_lens[b];
    if (kv_len > max_kv_len || kv_len < 0) {          // the block table holds max_kv_len keys at most
        if (pg == 0 && threadIdx.x == 0) record_status(status, KESSIE_DEV_BAD_ARG);
        kv_len = kv_len < 0 ? 0 : max_kv_len;
    }
    const int kv_pad = min(kv_max, (kv_len + 127) / 128 * 128);
    const int t0 = pg * ps;
    if (t0 >= kv_pad) return;
    int id = -1;
    if (t0 < kv_len) {
        id = bt[(int64_t)b * bt_stride + pg];
        if (id < 0 || id >= num_pages) {
            if (threadIdx.x == 0) record_status(status, KESSIE_DEV_BAD_PAGE_ID);
            id = -1;
        }
    }
    const int cs = (clear_start && fog_alpha > 0.f) ? clear_start[b] : INT_MIN;
    const bool has_fog = fog_w != nullptr || cs > 0;
    if (has_fog) {
        for (int s = threadIdx.x; s < ps; s += blockDim.x) {
            const int j = t0 + s;
            float w = 1.f;
            if (j >= kv_len) w = 0.f;
            else if (fog_w) w = __ldg(fog_w + b * fog_w_sb + j);
            else if (j < cs) {
                const float t = __fdiv_rn((float)j, (float)max(cs - 1, 1));
                w = fog_alpha == 0.5f ? sqrtf(t) : powf(t, fog_alpha);
            }
            wts[s] = w;
        }
        __syncthreads();
    }
    const int chunks = D / 8;
    const int items = 2 * Hkv * chunks;
    for (int it = threadIdx.x; it < items; it += blockDim.x) {
        const int kv = it / (Hkv * chunks);
        const int r = it - kv * Hkv * chunks;
        const int h = r / chunks, c = r - h * chunks;
        const T* src = (kv ? vc : kc) + (int64_t)(id < 0 ? 0 : id) * page_stride + (int64_t)h * head_stride + c * 8;
        T* dst = (kv ? sv : sk) + (((int64_t)b * Hkv + h) * kv_max + t0) * D + c * 8;
        const bool scale = kv && has_fog;
        for (int s = 0; s < ps && t0 + s < kv_pad; ++s) {
            uint4 v = make_uint4(0, 0, 0, 0);
            if (id >= 0 && t0 + s < kv_len) v = ldg_stream(src + (int64_t)s * token_stride);
            if (scale) {
                const float w = wts[s];
                T* e = reinterpret_cast<T*>(&v);
#pragma unroll
                for (int i = 0; i < 8; ++i) e[i] = from_f32<T>(to_f32(e[i]) * w);
            }
            *reinterpret_cast<uint4*>(dst + (int64_t)s * D) = v;
        }
    }
}

// Legacy dense [B,H,N,D] fp16 entry (kessie_kernels_v2.hip:716-751 / :788-825).
void legacy_dense(const void* Q, const void* K, const void* V, void* O, const void* fog, float sm_scale, int B, int H,
                  int N, int D, int W, int causal, void* stream, const char* name) {
    if (!Q || !K || !V || !O || B <= 0 || H <= 0 || N <= 0) {
        set_error(KESSIE_ERR_ARG, "%s: bad arguments", name);
        return;
    }
    if (D != 64 && D != 128) {
        set_error(KESSIE_ERR_UNSUPPORTED, "%s: head_dim=%d unsupported (64 or 128)", name, D);
        return;
    }
    PrefillParams p{};
    const int64_t sb = (int64_t)H * N * D, sh = (int64_t)N * D;
    p.q = Q; p.q_sb = sb; p.q_st = D; p.q_sh = sh;
    p.o = O; p.o_sb = sb; p.o_st = D; p.o_sh = sh;
    p.block_table = nullptr; p.bt_stride = 0;
    p.kv_lens = nullptr; p.kv_len_const = N;
    p.q_start = nullptr; p.q_start_const = 0;
    p.Nq = N; p.causal = causal ? 1 : 0; p.window = W > 0 ? W : 0;
    p.clear_start = nullptr; p.clear_start_const = 0; p.fog_alpha = 0.f;
    p.fog_w = static_cast<const float*>(fog); p.fog_w_sb = 0;
    p.scale_log2 = sm_scale * kLog2e;
    p.B = B; p.Hq = H; p.Hkv = H; p.G = 1; p.upp = 1; p.num_pages = B;
    p.status = device_status_ptr();
    run_prefill(p, K, V, sb, D, sh, B, N, D, false, as_stream(stream));
}

}  // namespace
}  // namespace kessie

using namespace kessie;

extern "C" void launch_kessie_windowed_attn(const void* Q, const void* K, const void* V, void* O, float sm_scale,
                                            int batch_size, int num_heads, int seq_len, int head_dim, int window_size,
                                            int is_causal, void* stream) {
    legacy_dense(Q, K, V, O, nullptr, sm_scale, batch_size, num_heads, seq_len, head_dim, window_size, is_causal,
                 stream, "launch_kessie_windowed_attn");
}

extern "C" void launch_kessie_fused_fog_attn(const void* Q, const void* K, const void* V, void* O,
                                             const void* fog_weights, float sm_scale, int batch_size, int num_heads,
                                             int seq_len, int head_dim, int window_size, int is_causal, void* stream) {
    if (!fog_weights) {
        set_error(KESSIE_ERR_ARG, "launch_kessie_fused_fog_attn: null fog_weights");
        return;
    }
    legacy_dense(Q, K, V, O, fog_weights, sm_scale, batch_size, num_heads, seq_len, head_dim, window_size, is_causal,
                 stream, "launch_kessie_fused_fog_attn");
}

extern "C" int kessie_fog_attention_v2(const void* q, const void* k, const void* v, void* out, int dtype,
                                       const float* fog_weights, float sm_scale, int batch, int num_q_heads,
                                       int num_kv_heads, int seq_len, int head_dim, int window_size, int is_causal,
                                       void* stream) {
    NvtxRange nvtx_range("kessie_fog_attention_v2");
    if (!dtype_ok(dtype)) return set_error(KESSIE_ERR_UNSUPPORTED, "fog_attention_v2: dtype %d", dtype);
    if (head_dim != 64 && head_dim != 128)
        return set_error(KESSIE_ERR_UNSUPPORTED, "fog_attention_v2: head_dim %d", head_dim);
    if (!q || !k || !v || !out || batch <= 0 || seq_len <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 ||
        num_q_heads % num_kv_heads)
        return set_error(KESSIE_ERR_ARG, "fog_attention_v2: bad arguments");
    if (dtype == KESSIE_DTYPE_F32) {
        // fp32 (the reference's own precision): every query row is one
        // "sequence" of the fp32 paged decode over this batch's K/V viewed as
        // 16-token pages (page p = tokens [16p, 16p + 16), head stride N*D);
        // one launch per batch, no workspace (a single split per row).
        if (num_q_heads / num_kv_heads > 16)
            return set_error(KESSIE_ERR_UNSUPPORTED, "fog_attention_v2: Hq/Hkv > 16 in fp32");
        if (((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15))
            return set_error(KESSIE_ERR_ARG, "fog_attention_v2: k/v must be 16-byte aligned");
        const int64_t sq = (int64_t)num_q_heads * seq_len * head_dim, skv = (int64_t)num_kv_heads * seq_len * head_dim;
        const int rows_per_launch = 65535 / num_kv_heads;        // grid y = rows x KV heads
        cudaStream_t st = as_stream(stream);
        for (int b = 0; b < batch; ++b)
        for (int r0 = 0; r0 < seq_len; r0 += rows_per_launch) {
            DecodeF32Args a{};
            a.q = static_cast<const float*>(q) + b * sq + (int64_t)r0 * head_dim;
            a.q_sb = head_dim; a.q_sh = (int64_t)seq_len * head_dim;
            a.k_cache = static_cast<const float*>(k) + b * skv;
            a.v_cache = static_cast<const float*>(v) + b * skv;
            a.page_stride = 16 * (int64_t)head_dim; a.token_stride = head_dim;
            a.head_stride = (int64_t)seq_len * head_dim;
            a.num_pages = (seq_len + 15) / 16; a.page_size = 16;
            a.fog_w = fog_weights; a.window = window_size > 0 ? window_size : 0; a.sm_scale = sm_scale;
            a.B = std::min(rows_per_launch, seq_len - r0); a.Hq = num_q_heads; a.Hkv = num_kv_heads; a.D = head_dim;
            a.max_seq_len = (seq_len + 15) / 16 * 16;
            a.slots = 0;                                   // one split per row: no workspace
            a.out = static_cast<float*>(out) + b * sq + (int64_t)r0 * head_dim;
            a.out_sb = head_dim; a.out_sh = (int64_t)seq_len * head_dim;
            a.status = device_status_ptr();
            a.square_n = seq_len; a.square_row0 = r0; a.causal = is_causal ? 1 : 0;
            const int rc = launch_decode_f32(a, st);
            if (rc) return rc;
        }
        return 0;
    }
    PrefillParams p{};
    const int64_t qsb = (int64_t)num_q_heads * seq_len * head_dim, ksb = (int64_t)num_kv_heads * seq_len * head_dim;
    const int64_t sh = (int64_t)seq_len * head_dim;
    p.q = q; p.q_sb = qsb; p.q_st = head_dim; p.q_sh = sh;
    p.o = out; p.o_sb = qsb; p.o_st = head_dim; p.o_sh = sh;
    p.kv_len_const = seq_len; p.Nq = seq_len; p.causal = is_causal ? 1 : 0; p.window = window_size > 0 ? window_size : 0;
    p.fog_w = fog_weights; p.scale_log2 = sm_scale * kLog2e;
    p.B = batch; p.Hq = num_q_heads; p.Hkv = num_kv_heads; p.G = num_q_heads / num_kv_heads; p.upp = 1; p.num_pages = batch;
    p.status = device_status_ptr();
    return run_prefill(p, k, v, ksb, head_dim, sh, batch, seq_len, head_dim, dtype == KESSIE_DTYPE_BF16, as_stream(stream));
}

extern "C" size_t kessie_paged_fog_prefill_workspace_size(int batch, int num_kv_heads, int head_dim, int max_kv_len) {
    if (batch <= 0 || num_kv_heads <= 0 || head_dim <= 0 || max_kv_len <= 0) return 0;
    const size_t kv_max = (size_t)(max_kv_len + 127) / 128 * 128;
    return 2 * (size_t)batch * num_kv_heads * kv_max * head_dim * 2 + 256;
}

namespace kessie {
namespace {
int prefill_entry(
    const void* q, int64_t q_stride_b, int64_t q_stride_t, int64_t q_stride_h, const void* k_cache, const void* v_cache,
    int64_t page_stride, int64_t token_stride, int64_t head_stride, int num_pages, int page_size,
    const int32_t* block_table, int64_t block_table_stride, const int32_t* kv_lens, const int32_t* q_start,
    const int32_t* clear_start, float fog_alpha, const float* fog_weights, int64_t fog_weights_stride_b,
    int window_size, int is_causal, float sm_scale, int batch, int num_q_tokens, int num_q_heads, int num_kv_heads,
    int head_dim, int dtype, const kessie_fog_bias* bias, void* out, int64_t o_stride_b, int64_t o_stride_t,
    int64_t o_stride_h, int max_kv_len, void* workspace, size_t workspace_bytes, void* stream) {
    NvtxRange nvtx_range("kessie_paged_fog_prefill");
    if (dtype != KESSIE_DTYPE_BF16 && dtype != KESSIE_DTYPE_F16)
        return set_error(KESSIE_ERR_UNSUPPORTED, "paged_fog_prefill_v2: dtype %d (f16/bf16 only)", dtype);
    if (head_dim != 64 && head_dim != 128)
        return set_error(KESSIE_ERR_UNSUPPORTED, "paged_fog_prefill_v2: head_dim %d", head_dim);
    if (page_size <= 0 || page_size % 16 || page_size > 256)
        return set_error(KESSIE_ERR_UNSUPPORTED, "paged_fog_prefill_v2: page_size %d", page_size);
    if (!q || !k_cache || !v_cache || !block_table || !kv_lens || !out || batch <= 0 || num_q_tokens < 0 ||
        num_q_heads <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads || num_pages <= 0)
        return set_error(KESSIE_ERR_ARG, "paged_fog_prefill_v2: bad arguments");
    if (((token_stride | head_stride | page_stride) & 7) || ((q_stride_t | q_stride_h | q_stride_b) & 1) ||
        ((o_stride_t | o_stride_h | o_stride_b) & 1))
        return set_error(KESSIE_ERR_ARG, "paged_fog_prefill_v2: misaligned strides");
    if (num_q_tokens == 0) { clear_error(); return 0; }
    PrefillParams p{};
    p.q = q; p.q_sb = q_stride_b; p.q_st = q_stride_t; p.q_sh = q_stride_h;
    p.o = out; p.o_sb = o_stride_b; p.o_st = o_stride_t; p.o_sh = o_stride_h;
    p.block_table = block_table; p.bt_stride = block_table_stride;
    p.kv_lens = kv_lens; p.q_start = q_start; p.q_start_const = -1;
    p.Nq = num_q_tokens; p.causal = is_causal ? 1 : 0; p.window = window_size > 0 ? window_size : 0;
    p.clear_start = clear_start; p.fog_alpha = fog_alpha; p.fog_w = fog_weights; p.fog_w_sb = fog_weights_stride_b;
    p.scale_log2 = sm_scale * kLog2e;
    p.B = batch; p.Hq = num_q_heads; p.Hkv = num_kv_heads; p.G = num_q_heads / num_kv_heads;
    p.upp = page_size / 16; p.num_pages = num_pages;
    p.status = device_status_ptr();
    int brc = fog_bias_from_c(bias, &p.bias);
    if (brc) return brc;
    const bool bf16 = dtype == KESSIE_DTYPE_BF16;
    cudaStream_t st = as_stream(stream);
    if (workspace && max_kv_len > 0 && head_dim % 8 == 0 && ((reinterpret_cast<uintptr_t>(workspace) & 15) == 0) &&
        ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15) == 0) {
        const size_t need = kessie_paged_fog_prefill_workspace_size(batch, num_kv_heads, head_dim, max_kv_len);
        if (workspace_bytes < need)
            return set_error(KESSIE_ERR_WORKSPACE, "paged_fog_prefill_ex_v2: workspace %zu < %zu", workspace_bytes, need);
        const int kv_max = (max_kv_len + 127) / 128 * 128;
        const size_t half = (size_t)batch * num_kv_heads * kv_max * head_dim;     // elements per K (or V)
        dim3 grid((kv_max + page_size - 1) / page_size, batch);
        if (bf16) {
            auto* sk = static_cast<__nv_bfloat16*>(workspace);
            stage_kv_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
                (const __nv_bfloat16*)k_cache, (const __nv_bfloat16*)v_cache, page_stride, token_stride, head_stride,
                num_pages, page_size, block_table, block_table_stride, kv_lens, max_kv_len, kv_max, num_kv_heads, head_dim,
                clear_start, fog_alpha, fog_weights, fog_weights_stride_b, sk, sk + half, p.status);
        } else {
            auto* sk = static_cast<__half*>(workspace);
            stage_kv_kernel<__half><<<grid, 256, 0, st>>>(
                (const __half*)k_cache, (const __half*)v_cache, page_stride, token_stride, head_stride, num_pages,
                page_size, block_table, block_table_stride, kv_lens, max_kv_len, kv_max, num_kv_heads, head_dim,
                clear_start, fog_alpha, fog_weights, fog_weights_stride_b, sk, sk + half, p.status);
        }
        int rc = check_launch("prefill staging");
        if (rc) return rc;
        // dense view of the staging buffer: page coordinate = sequence, token =
        // position; the fog weights are already in the staged V
        p.block_table = nullptr;
        p.num_pages = batch;
        p.clear_start = nullptr; p.clear_start_const = 0; p.fog_alpha = 0.f;
        p.fog_w = nullptr; p.fog_w_sb = 0;
        const char* base = static_cast<const char*>(workspace);
        return run_prefill(p, base, base + half * 2, (int64_t)num_kv_heads * kv_max * head_dim, head_dim,
                           (int64_t)kv_max * head_dim, batch, kv_max, head_dim, bf16, st);
    }
    return run_prefill(p, k_cache, v_cache, page_stride, token_stride, head_stride, num_pages, page_size, head_dim,
                       bf16, st);
}
}  // namespace
}  // namespace kessie

extern "C" int kessie_paged_fog_prefill_ex_v2(
    const void* q, int64_t q_stride_b, int64_t q_stride_t, int64_t q_stride_h, const void* k_cache, const void* v_cache,
    int64_t page_stride, int64_t token_stride, int64_t head_stride, int num_pages, int page_size,
    const int32_t* block_table, int64_t block_table_stride, const int32_t* kv_lens, const int32_t* q_start,
    const int32_t* clear_start, float fog_alpha, const float* fog_weights, int64_t fog_weights_stride_b,
    int window_size, int is_causal, float sm_scale, int batch, int num_q_tokens, int num_q_heads, int num_kv_heads,
    int head_dim, int dtype, void* out, int64_t o_stride_b, int64_t o_stride_t, int64_t o_stride_h, int max_kv_len,
    void* workspace, size_t workspace_bytes, void* stream) {
    return prefill_entry(q, q_stride_b, q_stride_t, q_stride_h, k_cache, v_cache, page_stride, token_stride,
                         head_stride, num_pages, page_size, block_table, block_table_stride, kv_lens, q_start,
                         clear_start, fog_alpha, fog_weights, fog_weights_stride_b, window_size, is_causal, sm_scale,
                         batch, num_q_tokens, num_q_heads, num_kv_heads, head_dim, dtype, nullptr, out, o_stride_b,
                         o_stride_t, o_stride_h, max_kv_len, workspace, workspace_bytes, stream);
}

extern "C" int kessie_paged_fog_prefill_biased_v2(
    const void* q, int64_t q_stride_b, int64_t q_stride_t, int64_t q_stride_h, const void* k_cache, const void* v_cache,
    int64_t page_stride, int64_t token_stride, int64_t head_stride, int num_pages, int page_size,
    const int32_t* block_table, int64_t block_table_stride, const int32_t* kv_lens, const int32_t* q_start,
    int window_size, int is_causal, float sm_scale, int batch, int num_q_tokens, int num_q_heads, int num_kv_heads,
    int head_dim, int dtype, const kessie_fog_bias* bias, void* out, int64_t o_stride_b, int64_t o_stride_t,
    int64_t o_stride_h, int max_kv_len, void* workspace, size_t workspace_bytes, void* stream) {
    return prefill_entry(q, q_stride_b, q_stride_t, q_stride_h, k_cache, v_cache, page_stride, token_stride,
                         head_stride, num_pages, page_size, block_table, block_table_stride, kv_lens, q_start, nullptr,
                         0.f, nullptr, 0, window_size, is_causal, sm_scale, batch, num_q_tokens, num_q_heads,
                         num_kv_heads, head_dim, dtype, bias, out, o_stride_b, o_stride_t, o_stride_h, max_kv_len,
                         workspace, workspace_bytes, stream);
}

extern "C" int kessie_paged_fog_prefill_v2(
    const void* q, int64_t q_stride_b, int64_t q_stride_t, int64_t q_stride_h, const void* k_cache, const void* v_cache,
    int64_t page_stride, int64_t token_stride, int64_t head_stride, int num_pages, int page_size,
    const int32_t* block_table, int64_t block_table_stride, const int32_t* kv_lens, const int32_t* q_start,
    const int32_t* clear_start, float fog_alpha, const float* fog_weights, int64_t fog_weights_stride_b,
    int window_size, int is_causal, float sm_scale, int batch, int num_q_tokens, int num_q_heads, int num_kv_heads,
    int head_dim, int dtype, void* out, int64_t o_stride_b, int64_t o_stride_t, int64_t o_stride_h, void* stream) {
    return kessie_paged_fog_prefill_ex_v2(q, q_stride_b, q_stride_t, q_stride_h, k_cache, v_cache, page_stride,
                                          token_stride, head_stride, num_pages, page_size, block_table,
                                          block_table_stride, kv_lens, q_start, clear_start, fog_alpha, fog_weights,
                                          fog_weights_stride_b, window_size, is_causal, sm_scale, batch, num_q_tokens,
                                          num_q_heads, num_kv_heads, head_dim, dtype, out, o_stride_b, o_stride_t,
                                          o_stride_h, 0, nullptr, 0, stream);
}
