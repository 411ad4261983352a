// fog_decode.cu -- paged fog-attention decode (split-KV) + log-sum-exp combine.
//
// Semantics: kessie_fused_fog_attention_ref (kessie_hip_kernels.py:577-593)
// at one query row per sequence, with GQA, a paged KV cache, per-sequence
// lengths and global positions (context-parallel shards):
//     O = sum_j p_j w_j v_j / sum_j p_j,  p_j = exp(q.k_j * sm_scale - m)
// over visible keys j (j <= q_pos, and q_pos - j < W when W > 0); the fog
// weight w_j scales V only -- the softmax denominator uses unweighted p
// (kessie_hip_kernels.py:152-158).
//
// Design (B200):
//   grid  = (chunk, kv_head, seq).  A chunk is `cu` 16-token units of one
//           sequence; each CTA streams its chunk's K/V once for all Hq/Hkv
//           query heads of its KV head (GQA), so every KV byte is read once.
//   CTA   = 1 producer warp + 4 consumer warps.  The producer's lane 0
//           prefetches the chunk's page ids into smem, then issues one TMA
//           tensor load per 16-token K (and V) slice into a 3-stage ring
//           (mbarrier full/empty pairs, bounded waits).  Tiles are 128-byte
//           swizzled so ldmatrix is conflict-free.
//   math  = consumer warp w takes unit (it*4 + w) of each stage:
//             S^T[16 keys x 8 q] = K[16 x D] . Q^T       (mma.sync m16n8k16)
//             online softmax per query column (shuffles over the 8 key rows)
//             P^T *= w_j (fog), movmatrix.trans -> B operand
//             O^T[D x 8 q] += V^T[D x 16] . P^T[16 x 8]   (ldmatrix.trans)
//           The GQA group sits in the N=8 dimension, so the tensor-core
//           tiles carry no padding rows for Hq/Hkv = 8.
//   merge = the 4 warps merge in smem; the CTA writes (O/l, m, l) for its
//           chunk; decode_combine_kernel merges chunks per (seq, q_head).
#include "common.cuh"
#include "ptx.cuh"
#include "tma_host.cuh"

#include <math.h>

#include <mutex>

namespace kessie {
namespace {

constexpr int kNCW = 4;          // consumer warps
constexpr int kNST = 3;          // pipeline stages
constexpr int kMaxCU = 512;      // max 16-token units per chunk
constexpr int kThreads = (kNCW + 1) * 32;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct DecodeParams {
    const void* q;
    int64_t q_sb, q_sh;
    const int32_t* block_table;
    int64_t bt_stride;
    const int32_t* seq_lens;
    const int32_t* kv_off;
    const int32_t* q_pos;
    const int32_t* clear_start;
    float fog_alpha;
    const float* fog_w;
    int window;
    float scale_log2;
    int B, Hq, Hkv, G;
    int units_per_page, num_pages, max_units, cu, max_chunks;
    float* part;          // [B][Hq][max_chunks][D+2]
    int* status;
};

// Visible local key range [k_lo, k_hi) of sequence b (shared with the combine).
__device__ __forceinline__ bool seq_range(const DecodeParams& p, int b, int& k_lo, int& k_hi, int& off) {
    int n = p.seq_lens[b];
    if (n < 0 || n > p.max_units * 16) {
        record_status(p.status, KESSIE_DEV_BAD_ARG);
        n = n < 0 ? 0 : p.max_units * 16;
    }
    off = p.kv_off ? p.kv_off[b] : 0;
    const int qp = p.q_pos ? p.q_pos[b] : off + n - 1;
    k_hi = min(n, qp - off + 1);
    k_lo = p.window > 0 ? max(0, qp - p.window + 1 - off) : 0;
    return k_hi > k_lo;
}

// Fog weight of the key at global position j (kessie_hip_kernels.py:408-412).
__device__ __forceinline__ float fog_weight(const DecodeParams& p, int cs, float inv_den, int j) {
    if (p.fog_w) return __ldg(p.fog_w + j);
    if (j >= cs) return 1.f;
    const float t = __fdiv_rn((float)j, (float)max(cs - 1, 1));
    return powf(t, p.fog_alpha);
}

template <int D>
struct Smem {
    static constexpr int kTile = 16 * D * 2;              // bytes of one 16-token K (or V) slice
    static constexpr int kStage = kNCW * 2 * kTile;
    static constexpr int kIdsOff = kNST * kStage;
    static constexpr int kBarOff = kIdsOff + kMaxCU * 4;
    static constexpr int kBytes = kBarOff + 2 * kNST * 8;
    static constexpr int kAlloc = kBytes + 1024;          // 1 KB slack for 1024-byte alignment
};

// Byte offset of (row r, 16B chunk c) inside a 128B-swizzled tile.
__device__ __forceinline__ uint32_t swz(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

template <int D, bool BF16, int NT>
__global__ void __launch_bounds__(kThreads, 2) fog_decode_kernel(const __grid_constant__ CUtensorMap tmK,
                                                                  const __grid_constant__ CUtensorMap tmV,
                                                                  const DecodeParams p) {
    using S = Smem<D>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    int32_t* ids = reinterpret_cast<int32_t*>(smem + S::kIdsOff);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kBarOff);
    uint64_t* empty = full + kNST;

    const int c = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
    int k_lo, k_hi, off;
    if (!seq_range(p, b, k_lo, k_hi, off)) return;
    const int u_lo = k_lo >> 4, u_hi = (k_hi + 15) >> 4;
    const int cu0 = max(u_lo, c * p.cu), cu1 = min(u_hi, (c + 1) * p.cu);
    if (cu1 <= cu0) return;
    const int nu = cu1 - cu0;
    const int n_iter = (nu + kNCW - 1) / kNCW;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kNST; ++s) { ptx::mbar_init(&full[s], 1); ptx::mbar_init(&empty[s], kNCW); }
        ptx::fence_mbar_init();
    }
    if (warp == kNCW) {
        const int32_t* bt = p.block_table + (int64_t)b * p.bt_stride;
        for (int i = lane; i < nu; i += 32) {
            int id = __ldg(bt + (cu0 + i) / p.units_per_page);
            if (id < 0 || id >= p.num_pages) { record_status(p.status, KESSIE_DEV_BAD_PAGE_ID); id = -1; }
            ids[i] = id;
        }
    }
    __syncthreads();

    // ------------------------------------------------------------ producer
    if (warp == kNCW) {
        if (lane == 0) {
            ptx::prefetch_tensormap(&tmK);
            ptx::prefetch_tensormap(&tmV);
            const uint64_t pol = ptx::policy_evict_first();
            int issued = 0;
            for (int it = 0; it < n_iter; ++it) {
                const int s = it % kNST;
                const uint32_t ph = (uint32_t)(it / kNST) & 1u;
                if (it >= kNST && !ptx::mbar_wait(&empty[s], ph ^ 1u)) {
                    record_status(p.status, KESSIE_DEV_WAIT_TIMEOUT);
                    break;
                }
                const int nu_it = min(kNCW, nu - it * kNCW);
                ptx::mbar_arrive_expect_tx(&full[s], (uint32_t)(nu_it * 2 * S::kTile));
                uint8_t* st = smem + s * S::kStage;
                for (int w = 0; w < nu_it; ++w) {
                    const int i = it * kNCW + w;
                    const int u = cu0 + i;
                    const int id = ids[i];
                    const int page = id < 0 ? p.num_pages : id;          // out of range -> zero fill
                    const int tok0 = (u % p.units_per_page) * 16;
                    ptx::tma_load_5d_hint(st + w * 2 * S::kTile, &tmK, &full[s], 0, tok0, 0, hk, page, pol);
                    ptx::tma_load_5d_hint(st + w * 2 * S::kTile + S::kTile, &tmV, &full[s], 0, tok0, 0, hk, page, pol);
                }
                issued = it + 1;
            }
            // drain: every issued load has landed before this thread exits
            for (int it = max(0, issued - kNST); it < issued; ++it) {
                if (!ptx::mbar_wait(&full[it % kNST], (uint32_t)(it / kNST) & 1u)) {
                    record_status(p.status, KESSIE_DEV_WAIT_TIMEOUT);
                    break;
                }
            }
        }
        return;
    }

    // ------------------------------------------------------------ consumers
    const int g = lane >> 2, t = lane & 3;
    // Q^T B-fragments: b0 = Q[q=g][kk*16+2t..+1], b1 = Q[g][kk*16+2t+8..+9]
    uint32_t qf[NT][D / 16][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int qh = nt * 8 + g;
        const bool ok = qh < p.G;
        const uint16_t* qrow = reinterpret_cast<const uint16_t*>(p.q) + (int64_t)b * p.q_sb +
                               (int64_t)(hk * p.G + (ok ? qh : 0)) * p.q_sh;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
            uint32_t lo = ok ? *reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 2 * t) : 0u;
            uint32_t hi = ok ? *reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 2 * t + 8) : 0u;
            qf[nt][kk][0] = lo;
            qf[nt][kk][1] = hi;
        }
    }
    float m[NT][2], l[NT][2], acc[NT][D / 16][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        m[nt][0] = m[nt][1] = -INFINITY;
        l[nt][0] = l[nt][1] = 0.f;
#pragma unroll
        for (int mt = 0; mt < D / 16; ++mt) acc[nt][mt][0] = acc[nt][mt][1] = acc[nt][mt][2] = acc[nt][mt][3] = 0.f;
    }
    const int cs = (p.clear_start && p.fog_alpha > 0.f) ? p.clear_start[b] : INT_MIN;
    const bool has_fog = p.fog_w != nullptr || cs > 0;

    // ldmatrix lane roles
    const int mi = lane >> 3, rr = lane & 7;
    // K (non-trans): key = rr + 8*(mi&1), chunk offset (mi>>1)
    const int k_key = rr + 8 * (mi & 1), k_cadd = mi >> 1;
    // V (trans): key = rr + 8*(mi>>1), chunk offset (mi&1)
    const int v_key = rr + 8 * (mi >> 1), v_cadd = mi & 1;

    bool timed_out = false;
    for (int it = 0; it < n_iter; ++it) {
        const int s = it % kNST;
        if (!ptx::mbar_wait(&full[s], (uint32_t)(it / kNST) & 1u)) {
            record_status(p.status, KESSIE_DEV_WAIT_TIMEOUT);
            timed_out = true;
            break;
        }
        const int i = it * kNCW + warp;
        if (i < nu) {
            uint8_t* ktile = smem + s * S::kStage + warp * 2 * S::kTile;
            uint8_t* vtile = ktile + S::kTile;
            const int u = cu0 + i;
            const int j0 = u * 16;                         // local index of key 0 of the unit
            const bool page_ok = ids[i] >= 0;
            const bool partial = (j0 < k_lo) || (j0 + 16 > k_hi) || !page_ok;
            if (partial) {
                // zero V rows of masked keys so 0 * (stale NaN) cannot leak into O
                for (int e = lane; e < 16 * (D / 64) * 8; e += 32) {
                    const int key = e & 15, dh = (e >> 4) % (D / 64), ch = e / (16 * (D / 64));
                    const int j = j0 + key;
                    if (!page_ok || j < k_lo || j >= k_hi)
                        *reinterpret_cast<uint4*>(vtile + swz(dh * 16 + key, ch)) = make_uint4(0, 0, 0, 0);
                }
                __syncwarp();
            }
            // ---- S^T = K . Q^T
            float sacc[NT][4];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.f;
            const uint32_t kb = ptx::smem_u32(ktile);
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
                const int chunk = kk * 2 + k_cadd;
                uint32_t a0, a1, a2, a3;
                ptx::ldmatrix_x4(a0, a1, a2, a3, kb + swz((chunk >> 3) * 16 + k_key, chunk & 7));
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) ptx::mma_16816<BF16>(sacc[nt], a0, a1, a2, a3, qf[nt][kk][0], qf[nt][kk][1]);
            }
            // ---- mask, online softmax, fog
            const int ja = j0 + g, jb = j0 + g + 8;
            const bool va = page_ok && ja >= k_lo && ja < k_hi;
            const bool vb = page_ok && jb >= k_lo && jb < k_hi;
            float wa = 1.f, wb = 1.f;
            if (has_fog) {      // only visible keys: fog_weights covers visible positions only
                wa = va ? fog_weight(p, cs, 0.f, off + ja) : 0.f;
                wb = vb ? fog_weight(p, cs, 0.f, off + jb) : 0.f;
            }
            uint32_t pb0[NT], pb1[NT];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const float s00 = va ? sacc[nt][0] * p.scale_log2 : -INFINITY;
                const float s01 = va ? sacc[nt][1] * p.scale_log2 : -INFINITY;
                const float s10 = vb ? sacc[nt][2] * p.scale_log2 : -INFINITY;
                const float s11 = vb ? sacc[nt][3] * p.scale_log2 : -INFINITY;
                float mx0 = fmaxf(s00, s10), mx1 = fmaxf(s01, s11);
#pragma unroll
                for (int o = 4; o < 32; o <<= 1) {
                    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
                    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
                }
                const float mn0 = fmaxf(m[nt][0], mx0), mn1 = fmaxf(m[nt][1], mx1);
                const float base0 = mn0 == -INFINITY ? 0.f : mn0;
                const float base1 = mn1 == -INFINITY ? 0.f : mn1;
                const float al0 = exp2f(m[nt][0] - base0), al1 = exp2f(m[nt][1] - base1);
                const float p00 = exp2f(s00 - base0), p01 = exp2f(s01 - base1);
                const float p10 = exp2f(s10 - base0), p11 = exp2f(s11 - base1);
                l[nt][0] = l[nt][0] * al0 + p00 + p10;
                l[nt][1] = l[nt][1] * al1 + p01 + p11;
                m[nt][0] = mn0;
                m[nt][1] = mn1;
#pragma unroll
                for (int mt = 0; mt < D / 16; ++mt) {
                    acc[nt][mt][0] *= al0; acc[nt][mt][1] *= al1;
                    acc[nt][mt][2] *= al0; acc[nt][mt][3] *= al1;
                }
                pb0[nt] = ptx::movmatrix_trans(ptx::pack2<BF16>(p00 * wa, p01 * wa));
                pb1[nt] = ptx::movmatrix_trans(ptx::pack2<BF16>(p10 * wb, p11 * wb));
            }
            // ---- O^T += V^T . P^T
            const uint32_t vb_addr = ptx::smem_u32(vtile);
#pragma unroll
            for (int mt = 0; mt < D / 16; ++mt) {
                const int chunk = mt * 2 + v_cadd;
                uint32_t a0, a1, a2, a3;
                ptx::ldmatrix_x4_trans(a0, a1, a2, a3, vb_addr + swz((chunk >> 3) * 16 + v_key, chunk & 7));
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) ptx::mma_16816<BF16>(acc[nt][mt], a0, a1, a2, a3, pb0[nt], pb1[nt]);
            }
            if (partial) ptx::fence_proxy_async_smem();
        }
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&empty[s]);
    }

    // ------------------------------------------------------------ merge the 4 warps
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) l[nt][j] += __shfl_xor_sync(0xffffffffu, l[nt][j], o);

    constexpr int QP = NT * 8;                      // padded queries
    float* mw = reinterpret_cast<float*>(smem);     // [kNCW][QP]
    float* lw = mw + kNCW * QP;                     // [kNCW][QP]
    float* ow = lw + kNCW * QP;                     // [kNCW][D][QP]
    asm volatile("bar.sync 1, %0;" :: "r"(kNCW * 32) : "memory");   // all consumers done with the ring
    if (!timed_out) {
        if (g == 0) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                mw[warp * QP + nt * 8 + 2 * t] = m[nt][0];
                mw[warp * QP + nt * 8 + 2 * t + 1] = m[nt][1];
                lw[warp * QP + nt * 8 + 2 * t] = l[nt][0];
                lw[warp * QP + nt * 8 + 2 * t + 1] = l[nt][1];
            }
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int mt = 0; mt < D / 16; ++mt) {
                float* o = ow + (warp * D + mt * 16 + g) * QP + nt * 8 + 2 * t;
                o[0] = acc[nt][mt][0];
                o[1] = acc[nt][mt][1];
                o[8 * QP] = acc[nt][mt][2];
                o[8 * QP + 1] = acc[nt][mt][3];
            }
    }
    asm volatile("bar.sync 1, %0;" :: "r"(kNCW * 32) : "memory");
    if (timed_out) return;
    const int tid = threadIdx.x;                    // 0..127
    for (int e = tid; e < p.G * (D + 2); e += kNCW * 32) {
        const int q = e / (D + 2), d = e - q * (D + 2);
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kNCW; ++w) M = fmaxf(M, mw[w * QP + q]);
        float L = 0.f, O = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < kNCW; ++w) {
                const float sc = exp2f(mw[w * QP + q] - M);
                L += lw[w * QP + q] * sc;
                if (d < D) O += ow[(w * D + d) * QP + q] * sc;
            }
        }
        float v = d < D ? (L > 0.f ? O / L : 0.f) : (d == D ? M : L);
        p.part[(((int64_t)b * p.Hq + hk * p.G + q) * p.max_chunks + c) * (D + 2) + d] = v;
    }
}

// Merge the chunk partials of one (seq, q_head) row; blockDim = D.
template <typename T>
__global__ void decode_combine_kernel(const DecodeParams p, int D, T* __restrict__ out, float* __restrict__ out_part) {
    const int row = blockIdx.x;                 // b * Hq + hq
    const int b = row / p.Hq;
    const int d = threadIdx.x;
    int k_lo, k_hi, off;
    float M = -INFINITY, L = 0.f, O = 0.f;
    if (seq_range(p, b, k_lo, k_hi, off)) {
        const int u_lo = k_lo >> 4, u_hi = (k_hi + 15) >> 4;
        const int c_lo = u_lo / p.cu, c_hi = (u_hi - 1) / p.cu + 1;
        const float* base = p.part + (int64_t)row * p.max_chunks * (D + 2);
        for (int c = c_lo; c < c_hi; ++c) M = fmaxf(M, base[c * (D + 2) + D]);
        if (M != -INFINITY) {
            for (int c = c_lo; c < c_hi; ++c) {
                const float* pc = base + c * (D + 2);
                const float w = pc[D + 1] * exp2f(pc[D] - M);
                L += w;
                O += w * pc[d];
            }
        }
    }
    const float o = L > 0.f ? O / L : 0.f;
    if (out) out[(int64_t)row * D + d] = from_f32<T>(o);
    if (out_part) {
        out_part[(int64_t)row * (D + 2) + d] = o;
        if (d == 0) {
            out_part[(int64_t)row * (D + 2) + D] = M == -INFINITY ? -INFINITY : M * kLn2;
            out_part[(int64_t)row * (D + 2) + D + 1] = L;
        }
    }
}

// Merge S partial triples (natural-log m) per row; blockDim = D.
template <typename T>
__global__ void lse_combine_kernel(const float* __restrict__ parts, int S, int64_t sstride, int D,
                                   T* __restrict__ out, float* __restrict__ out_part) {
    const int row = blockIdx.x, d = threadIdx.x;
    float M = -INFINITY;
    for (int s = 0; s < S; ++s) M = fmaxf(M, parts[s * sstride + (int64_t)row * (D + 2) + D]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
        for (int s = 0; s < S; ++s) {
            const float* pr = parts + s * sstride + (int64_t)row * (D + 2);
            const float w = pr[D + 1] * __expf(pr[D] - M);
            L += w;
            O += w * pr[d];
        }
    }
    const float o = L > 0.f ? O / L : 0.f;
    if (out) out[(int64_t)row * D + d] = from_f32<T>(o);
    if (out_part) {
        out_part[(int64_t)row * (D + 2) + d] = o;
        if (d == 0) {
            out_part[(int64_t)row * (D + 2) + D] = M;
            out_part[(int64_t)row * (D + 2) + D + 1] = L;
        }
    }
}

struct Plan { int cu, max_units, max_chunks; size_t ws; };

Plan make_plan(int B, int Hq, int Hkv, int D, int max_seq_len) {
    Plan pl;
    pl.max_units = (max_seq_len + 15) / 16;
    if (pl.max_units < 1) pl.max_units = 1;
    const long long tot = (long long)B * Hkv * pl.max_units;
    const long long slots = (long long)sm_count() * 2;
    long long cu = (tot + slots * 8 - 1) / (slots * 8);
    cu = (cu + kNCW - 1) / kNCW * kNCW;
    if (cu < 16) cu = 16;
    if (cu > kMaxCU) cu = kMaxCU;
    pl.cu = (int)cu;
    pl.max_chunks = (pl.max_units + pl.cu - 1) / pl.cu;
    pl.ws = align_up((size_t)B * Hq * pl.max_chunks * (D + 2) * sizeof(float), 256);
    return pl;
}

template <int D, bool BF16, int NT>
int launch_decode_t(const CUtensorMap& mk, const CUtensorMap& mv, const DecodeParams& p, cudaStream_t st) {
    auto kern = fog_decode_kernel<D, BF16, NT>;
    const int smem = Smem<D>::kAlloc;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
        return check_launch("decode: set smem attribute");
    dim3 grid(p.max_chunks, p.Hkv, p.B);
    kern<<<grid, kThreads, smem, st>>>(mk, mv, p);
    return check_launch("paged_fog_decode");
}

}  // namespace
}  // namespace kessie

using namespace kessie;

extern "C" size_t kessie_paged_fog_decode_workspace_size(int batch, int num_q_heads, int num_kv_heads, int head_dim,
                                                         int max_seq_len, int page_size) {
    (void)page_size;
    if (batch <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0) return 0;
    return make_plan(batch, num_q_heads, num_kv_heads, head_dim, max_seq_len).ws;
}

extern "C" int kessie_paged_fog_decode_ex_v2(
    const void* q, int64_t q_stride_b, int64_t q_stride_h, const void* k_cache, const void* v_cache,
    int64_t page_stride, int64_t token_stride, int64_t head_stride, int num_pages, int page_size,
    const int32_t* block_table, int64_t block_table_stride, const int32_t* seq_lens, const int32_t* kv_pos_offset,
    const int32_t* q_positions, const int32_t* clear_start, float fog_alpha, const float* fog_weights,
    int window_size, float sm_scale, int batch, int num_q_heads, int num_kv_heads, int head_dim, int max_seq_len,
    int dtype, void* out, float* out_partial, void* workspace, size_t workspace_bytes, int phases, void* stream) {
    if (dtype != KESSIE_DTYPE_BF16 && dtype != KESSIE_DTYPE_F16)
        return set_error(KESSIE_ERR_UNSUPPORTED, "paged_fog_decode_v2: dtype %d (f16/bf16 only)", dtype);
    if (head_dim != 64 && head_dim != 128)
        return set_error(KESSIE_ERR_UNSUPPORTED, "paged_fog_decode_v2: head_dim %d (64/128 only)", head_dim);
    if (batch <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads)
        return set_error(KESSIE_ERR_ARG, "paged_fog_decode_v2: bad head counts Hq=%d Hkv=%d", num_q_heads, num_kv_heads);
    const int G = num_q_heads / num_kv_heads;
    if (G > 16) return set_error(KESSIE_ERR_UNSUPPORTED, "paged_fog_decode_v2: Hq/Hkv=%d > 16", G);
    if (page_size <= 0 || page_size % 16 || page_size > 256)
        return set_error(KESSIE_ERR_UNSUPPORTED, "paged_fog_decode_v2: page_size %d (multiple of 16, <= 256)", page_size);
    if (phases < 1 || phases > 3) return set_error(KESSIE_ERR_ARG, "paged_fog_decode_v2: phases %d", phases);
    if (!q || !k_cache || !v_cache || !block_table || !seq_lens || ((phases & 2) && !out && !out_partial) ||
        num_pages <= 0 || max_seq_len < 0)
        return set_error(KESSIE_ERR_ARG, "paged_fog_decode_v2: null pointer or bad size");
    if ((q_stride_h & 1) || (q_stride_b & 1) || (reinterpret_cast<uintptr_t>(q) & 3))
        return set_error(KESSIE_ERR_ARG, "paged_fog_decode_v2: q rows must be 4-byte aligned");
    if (((token_stride | head_stride | page_stride) & 7) || (reinterpret_cast<uintptr_t>(k_cache) & 15) ||
        (reinterpret_cast<uintptr_t>(v_cache) & 15))
        return set_error(KESSIE_ERR_ARG, "paged_fog_decode_v2: cache strides/base must be 16-byte multiples");
    Plan pl = make_plan(batch, num_q_heads, num_kv_heads, head_dim, max_seq_len);
    if (!workspace || workspace_bytes < pl.ws)
        return set_error(KESSIE_ERR_WORKSPACE, "paged_fog_decode_v2: workspace %zu < %zu", workspace_bytes, pl.ws);
    if (pl.max_chunks > 65535 * 16) return set_error(KESSIE_ERR_UNSUPPORTED, "paged_fog_decode_v2: too many chunks");

    const bool bf16 = dtype == KESSIE_DTYPE_BF16;
    DecodeParams p;
    p.q = q; p.q_sb = q_stride_b; p.q_sh = q_stride_h;
    p.block_table = block_table; p.bt_stride = block_table_stride;
    p.seq_lens = seq_lens; p.kv_off = kv_pos_offset; p.q_pos = q_positions; p.clear_start = clear_start;
    p.fog_alpha = fog_alpha; p.fog_w = fog_weights;
    p.window = window_size;
    p.scale_log2 = sm_scale * kLog2e;
    p.B = batch; p.Hq = num_q_heads; p.Hkv = num_kv_heads; p.G = G;
    p.units_per_page = page_size / 16; p.num_pages = num_pages;
    p.max_units = pl.max_units; p.cu = pl.cu; p.max_chunks = pl.max_chunks;
    p.part = static_cast<float*>(workspace);
    p.status = device_status_ptr();
    cudaStream_t st = as_stream(stream);

    if (phases & 1) {
        CUtensorMap mk, mv;
        CUresult r1 = encode_kv_tile_map(&mk, k_cache, bf16, head_dim, page_size, num_kv_heads, num_pages,
                                         token_stride, head_stride, page_stride);
        CUresult r2 = encode_kv_tile_map(&mv, v_cache, bf16, head_dim, page_size, num_kv_heads, num_pages,
                                         token_stride, head_stride, page_stride);
        if (r1 != CUDA_SUCCESS || r2 != CUDA_SUCCESS)
            return set_error(KESSIE_ERR_ARG, "paged_fog_decode_v2: TMA descriptor rejected (%d/%d)", (int)r1, (int)r2);
        int rc;
        const bool nt2 = G > 8;
        if (head_dim == 128) {
            if (bf16) rc = nt2 ? launch_decode_t<128, true, 2>(mk, mv, p, st) : launch_decode_t<128, true, 1>(mk, mv, p, st);
            else rc = nt2 ? launch_decode_t<128, false, 2>(mk, mv, p, st) : launch_decode_t<128, false, 1>(mk, mv, p, st);
        } else {
            if (bf16) rc = nt2 ? launch_decode_t<64, true, 2>(mk, mv, p, st) : launch_decode_t<64, true, 1>(mk, mv, p, st);
            else rc = nt2 ? launch_decode_t<64, false, 2>(mk, mv, p, st) : launch_decode_t<64, false, 1>(mk, mv, p, st);
        }
        if (rc) return rc;
    }
    if (phases & 2) {
        const int rows = batch * num_q_heads;
        if (bf16) decode_combine_kernel<__nv_bfloat16><<<rows, head_dim, 0, st>>>(p, head_dim, (__nv_bfloat16*)out, out_partial);
        else decode_combine_kernel<__half><<<rows, head_dim, 0, st>>>(p, head_dim, (__half*)out, out_partial);
        return check_launch("paged_fog_decode combine");
    }
    clear_error();
    return 0;
}

extern "C" int kessie_paged_fog_decode_v2(
    const void* q, int64_t q_stride_b, int64_t q_stride_h, const void* k_cache, const void* v_cache,
    int64_t page_stride, int64_t token_stride, int64_t head_stride, int num_pages, int page_size,
    const int32_t* block_table, int64_t block_table_stride, const int32_t* seq_lens, const int32_t* kv_pos_offset,
    const int32_t* q_positions, const int32_t* clear_start, float fog_alpha, const float* fog_weights,
    int window_size, float sm_scale, int batch, int num_q_heads, int num_kv_heads, int head_dim, int max_seq_len,
    int dtype, void* out, float* out_partial, void* workspace, size_t workspace_bytes, void* stream) {
    return kessie_paged_fog_decode_ex_v2(q, q_stride_b, q_stride_h, k_cache, v_cache, page_stride, token_stride,
                                         head_stride, num_pages, page_size, block_table, block_table_stride, seq_lens,
                                         kv_pos_offset, q_positions, clear_start, fog_alpha, fog_weights, window_size,
                                         sm_scale, batch, num_q_heads, num_kv_heads, head_dim, max_seq_len, dtype, out,
                                         out_partial, workspace, workspace_bytes, 3, stream);
}

extern "C" int kessie_lse_combine_v2(const float* partials, int num_splits, int64_t split_stride, int rows,
                                     int head_dim, void* out, int out_dtype, float* out_partial, void* stream) {
    if (!partials || num_splits <= 0 || rows <= 0 || head_dim <= 0 || head_dim > 1024 || (!out && !out_partial))
        return set_error(KESSIE_ERR_ARG, "lse_combine_v2: bad arguments");
    if (!dtype_ok(out_dtype)) return set_error(KESSIE_ERR_UNSUPPORTED, "lse_combine_v2: dtype %d", out_dtype);
    cudaStream_t st = as_stream(stream);
    switch (out_dtype) {
        case KESSIE_DTYPE_F16: lse_combine_kernel<__half><<<rows, head_dim, 0, st>>>(partials, num_splits, split_stride, head_dim, (__half*)out, out_partial); break;
        case KESSIE_DTYPE_BF16: lse_combine_kernel<__nv_bfloat16><<<rows, head_dim, 0, st>>>(partials, num_splits, split_stride, head_dim, (__nv_bfloat16*)out, out_partial); break;
        default: lse_combine_kernel<float><<<rows, head_dim, 0, st>>>(partials, num_splits, split_stride, head_dim, (float*)out, out_partial); break;
    }
    return check_launch("lse_combine");
}

// ============================================================================
// Allocation-free decode entry point.
//
// Some callers cannot allocate device memory at the point where they decode:
// code running under an allocator that is frozen or owned by someone else
// (a serving engine that pre-reserved all of HBM for its KV pool, a plugin
// invoked from inside another runtime's step, a process that must not grow
// its footprint after start-up).  They cannot provide the split-KV scratch
// that kessie_paged_fog_decode_v2 takes as `workspace`.  This variant keeps
// that scratch in a fixed array inside the library instead.
//
// The array below is file-scope device memory of KESSIE_NOALLOC_SCRATCH_BYTES
// (16 MiB); every GPU that loads this library holds it until the process
// exits.  Its name is only a host-side handle: host code must never pass it
// to a kernel.  Its device address is looked up with cudaGetSymbolAddress
// once per device, on the first call made with that device current, and
// cached; make that first call before any stream capture.  All calls share
// the one array, so two calls whose work overlaps on the GPU (different
// streams, or different threads using one device) race on it; callers must
// order them.  The array keeps whatever the previous call left: the decode
// writes every partial it later reads, so nothing needs clearing.
// ============================================================================
namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[KESSIE_NOALLOC_SCRATCH_BYTES];

constexpr int kNoAllocMaxDevices = 64;
void* g_noalloc_ptr[kNoAllocMaxDevices] = {nullptr};
std::mutex g_noalloc_mu;

// Device address of g_noalloc_scratch on the current device (set-up on first use).
int noalloc_scratch(void** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return set_error(KESSIE_ERR_CUDA, "noalloc decode: cudaGetDevice failed");
    if (dev < 0 || dev >= kNoAllocMaxDevices) return set_error(KESSIE_ERR_UNSUPPORTED, "noalloc decode: device %d", dev);
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p)
            return set_error(KESSIE_ERR_CUDA, "noalloc decode: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return KESSIE_OK;
}

}  // namespace

extern "C" int kessie_paged_fog_decode_noalloc_v2(
    const void* q, int64_t q_stride_b, int64_t q_stride_h, const void* k_cache, const void* v_cache,
    int64_t page_stride, int64_t token_stride, int64_t head_stride, int num_pages, int page_size,
    const int32_t* block_table, int64_t block_table_stride, const int32_t* seq_lens, const int32_t* kv_pos_offset,
    const int32_t* q_positions, const int32_t* clear_start, float fog_alpha, const float* fog_weights,
    int window_size, float sm_scale, int batch, int num_q_heads, int num_kv_heads, int head_dim, int max_seq_len,
    int dtype, void* out, float* out_partial, void* stream) {
    if (batch <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 || max_seq_len < 0)
        return set_error(KESSIE_ERR_ARG, "noalloc decode: bad sizes");
    const size_t need = kessie_paged_fog_decode_workspace_size(batch, num_q_heads, num_kv_heads, head_dim,
                                                               max_seq_len, page_size);
    if (need > (size_t)KESSIE_NOALLOC_SCRATCH_BYTES)
        return set_error(KESSIE_ERR_WORKSPACE,
                         "noalloc decode: this shape needs %zu bytes of scratch, above the built-in %d-byte array; "
                         "use kessie_paged_fog_decode_v2 with a caller-provided workspace",
                         need, (int)KESSIE_NOALLOC_SCRATCH_BYTES);
    void* scratch = nullptr;
    int rc = noalloc_scratch(&scratch);
    if (rc) return rc;
    return kessie_paged_fog_decode_ex_v2(q, q_stride_b, q_stride_h, k_cache, v_cache, page_stride, token_stride,
                                         head_stride, num_pages, page_size, block_table, block_table_stride, seq_lens,
                                         kv_pos_offset, q_positions, clear_start, fog_alpha, fog_weights, window_size,
                                         sm_scale, batch, num_q_heads, num_kv_heads, head_dim, max_seq_len, dtype, out,
                                         out_partial, scratch, (size_t)KESSIE_NOALLOC_SCRATCH_BYTES, 3, stream);
}
