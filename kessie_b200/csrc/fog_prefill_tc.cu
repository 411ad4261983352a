// fog_prefill_tc.cu -- chunked-prefill fog attention on the 5th-generation
// tensor cores (tcgen05 + TMEM), head_dim 128, bf16 / fp16.
//
// Semantics are those of fog_prefill.cu (kessie_hip_kernels.py:577-593 with a
// query offset, GQA, paged or dense KV): O_i = sum_j p_ij w_j v_j / sum_j p_ij.
//
// CTA = two 128-row Q tiles (A, B) of one KV head -- rows are (token,
// head-in-group) pairs, so the Hq/Hkv heads sharing a KV head share every K/V
// tile -- and 12 warps:
//   warps 0-3 / 4-7  softmax warpgroups, one per Q tile, one row per thread
//              (TMEM lane = row): tcgen05.ld S, mask (boundary tiles only),
//              online max, p = 2^(s*scale - m) with packed fp32 pairs, row sum
//              of p, P = p (or p * w when the fog is applied in-kernel: the
//              staged path folds the fog weights into V), tcgen05.st P.  The
//              running max moves (and O is rescaled in TMEM, after P) only
//              when it grows by more than 2^8.
//   warp 8     Q loader, then the K producer: 128-key K tiles (one TMA box per
//              d-half) into a 2-stage ring.
//   warp 9     TMEM owner (512 columns) and MMA issuer (one thread), per KV
//              tile t:  PV_A(t) S_A(t+1) PV_B(t) S_B(t+1), where
//                S_X  = Q_X K^T     tcgen05.mma SS, M128 N128 K16 x 8
//                O_X += P_X V       tcgen05.mma TS (P in TMEM), V MN-major
//              so the tensor core computes one tile's scores while the other
//              tile's softmax runs.
//   warp 10    V producer: 128-key V tiles into a 2-stage ring.
//   warp 11    idle (keeps the producer warpgroup whole for setmaxnreg).
// TMEM columns: S_A [0,128) S_B [128,256) O_A [256,384) O_B [384,512); P_X
// (16-bit pairs) overwrites the first 64 columns of S_X.
// setmaxnreg: the producer warpgroup drops to 64 registers, the softmax
// warpgroups rise to 216 (launch 168; the host checks the launch pool).
// Every mbarrier wait is bounded; on a timeout all warps still reach the
// final barrier and the TMEM is freed.
#include "common.cuh"
#include "ptx.cuh"
#include "tma_host.cuh"
#include "prefill_common.cuh"

#include <math.h>
#include <stdlib.h>
#include <string.h>

namespace kessie {
namespace {

constexpr int kNK = 2;                 // K stages
constexpr int kNV = 2;                 // V stages
constexpr int kThreads = 384;          // warps 0-7: softmax A / B; 8: K producer; 9: MMA; 10: V producer; 11: idle
// setmaxnreg split: the launch pool is kThreads x kLaunchRegs; the producer
// warpgroup gives registers back to the two softmax warpgroups.
constexpr int kLaunchRegs = 168, kSoftmaxRegs = 216, kProducerRegs = 64;
static_assert(256 * kSoftmaxRegs + 128 * kProducerRegs <= kThreads * kLaunchRegs, "register split exceeds the pool");
constexpr int kRowsPerCta = 256;       // two 128-row Q tiles (A, B)
constexpr uint32_t kTmemCols = 512;    // S_A [0,128) S_B [128,256) O_A [256,384) O_B [384,512)
constexpr float kRescaleThreshold = 8.0f;    // log2 units
constexpr float kLog2eTc = 1.4426950408889634f;

struct L {
    static constexpr int kHalf = 128 * 128;         // [128 rows][64 el] x 2 B
    static constexpr int kTile = 2 * kHalf;         // both d-halves: 32 KB
    static constexpr int kQ = 0;                    // Q_A, Q_B
    static constexpr int kK = kQ + 2 * kTile;
    static constexpr int kV = kK + kNK * kTile;
    static constexpr int kW = kV + kNV * kTile;     // per softmax warp: fog weights of the tile's 128 keys
    static constexpr int kB = kW + 8 * 128 * 4;     // per softmax warp: additive bias / sm_scale of those keys
    static constexpr int kBar = kB + 8 * 128 * 4;
    // q_full, k_full[NK], k_empty[NK], v_full[NV], v_empty[NV], s_full[2], p_full[2], o_bar[2]
    static constexpr int kNumBar = 1 + 2 * kNK + 2 * kNV + 6;
    static constexpr int kSlot = kBar + kNumBar * 8;
    static constexpr int kBytes = kSlot + 16;
    static constexpr int kAlloc = kBytes + 1024;
};

struct TcArgs {
    PrefillParams p;
    int q_mode;        // 0: Q map {64, g, t(batch-folded), dh, hk}; 1: {64, t, dh, h, b} (G == 1)
    int box_tokens;    // tokens per K/V box
    int dense;         // K/V map page coordinate = batch
    int page_size;
};

// P of one 128-key tile for one row: p = 2^(s*scale - m), P' = p * w (FOG:
// the fog weights of the tile's keys in wbuf; the staged path carries them in
// V instead, and then key pairs go through packed fp32 arithmetic -- one fma
// and one add instruction per pair, the exponentials on the MUFU), packed to
// 16-bit pairs over the first 64 columns of the row's S region.  Returns the
// row sum of the unweighted p.  Warp-collective (tcgen05.st).
template <bool BF16, bool FOG>
__device__ __forceinline__ float softmax_p_tile(const uint32_t (&sv)[4][32], uint32_t sreg, float scale_log2,
                                                float nb, const float* wbuf) {
    float lsum;
    if (FOG) {
        // scalar form: the weights' registers leave no room for packed pairs
        const float4* w4 = reinterpret_cast<const float4*>(wbuf);
        float lt4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int h4 = 0; h4 < 4; ++h4) {
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; i += 2) {
                const float4 w = w4[(h4 * 32 + 2 * i) >> 2];      // keys h4*32 + 2i .. +3
                const float p0 = ptx::ex2(fmaf(__uint_as_float(sv[h4][2 * i]), scale_log2, nb));
                const float p1 = ptx::ex2(fmaf(__uint_as_float(sv[h4][2 * i + 1]), scale_log2, nb));
                const float p2 = ptx::ex2(fmaf(__uint_as_float(sv[h4][2 * i + 2]), scale_log2, nb));
                const float p3 = ptx::ex2(fmaf(__uint_as_float(sv[h4][2 * i + 3]), scale_log2, nb));
                lt4[0] += p0; lt4[1] += p1; lt4[2] += p2; lt4[3] += p3;
                pk[i] = ptx::pack2<BF16>(p0 * w.x, p1 * w.y);
                pk[i + 1] = ptx::pack2<BF16>(p2 * w.z, p3 * w.w);
            }
            ptx::tmem_st16(sreg + h4 * 16, pk);
        }
        lsum = (lt4[0] + lt4[1]) + (lt4[2] + lt4[3]);
    } else {
        const uint64_t sc2 = ptx::f2_pack(scale_log2, scale_log2), nb2 = ptx::f2_pack(nb, nb);
        uint64_t lt2[2] = {0ull, 0ull};
#pragma unroll
        for (int h4 = 0; h4 < 4; ++h4) {
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const uint64_t s2 = ptx::f2_pack(__uint_as_float(sv[h4][2 * i]), __uint_as_float(sv[h4][2 * i + 1]));
                float e0, e1;
                ptx::f2_unpack(ptx::ffma2(s2, sc2, nb2), e0, e1);
                const float p0 = ptx::ex2(e0), p1 = ptx::ex2(e1);
                lt2[i & 1] = ptx::fadd2(lt2[i & 1], ptx::f2_pack(p0, p1));
                pk[i] = ptx::pack2<BF16>(p0, p1);
            }
            ptx::tmem_st16(sreg + h4 * 16, pk);
        }
        float a0, a1, b0, b1;
        ptx::f2_unpack(lt2[0], a0, a1);
        ptx::f2_unpack(lt2[1], b0, b1);
        lsum = (a0 + a1) + (b0 + b1);
    }
    ptx::tmem_st_wait();
    return lsum;
}

template <bool BF16>
__global__ void __launch_bounds__(kThreads, 1) fog_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                                                                      const __grid_constant__ CUtensorMap tmK,
                                                                      const __grid_constant__ CUtensorMap tmV,
                                                                      const TcArgs a) {
    const PrefillParams& p = a.p;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
    uint64_t* q_full = bars;
    uint64_t* k_full = bars + 1;
    uint64_t* k_empty = k_full + kNK;
    uint64_t* v_full = k_empty + kNK;
    uint64_t* v_empty = v_full + kNV;
    uint64_t* s_full = v_empty + kNV;      // [2]: Q tile A, B
    uint64_t* p_full = s_full + 2;
    uint64_t* o_bar = p_full + 2;
    uint32_t* slot = reinterpret_cast<uint32_t*>(smem + L::kSlot);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile_m = gridDim.x - 1 - blockIdx.x;          // heavy (late, causal) row tiles first
    const int hk = blockIdx.y, b = blockIdx.z;
    const int G = p.G;
    const int rows_total = p.Nq * G;
    const int row0 = tile_m * kRowsPerCta;
    const int kv_len = p.kv_lens ? p.kv_lens[b] : p.kv_len_const;
    const int q0 = p.q_start ? p.q_start[b] : (p.q_start_const >= 0 ? p.q_start_const : kv_len - p.Nq);
    const int t_first = row0 / G;
    const int t_last = (min(row0 + kRowsPerCta, rows_total) - 1) / G;
    const int pos_lo = q0 + t_first, pos_hi = q0 + t_last;
    int j_lo = p.window > 0 ? max(0, pos_lo - p.window + 1) : 0;
    int j_hi = (p.causal || p.window > 0) ? min(kv_len, pos_hi + 1) : kv_len;
    if (j_hi < j_lo) j_hi = j_lo;
    const int tile_lo = j_lo / 128, tile_hi = (j_hi + 127) / 128;
    const int n_tiles = tile_hi - tile_lo;
    const int cs = (p.clear_start || p.clear_start_const > 0) && p.fog_alpha > 0.f
                       ? (p.clear_start ? p.clear_start[b] : p.clear_start_const) : INT_MIN;
    const bool has_fog = p.fog_w != nullptr || cs > 0;

    if (threadIdx.x == 0) {
        ptx::mbar_init(q_full, 1);
        for (int i = 0; i < kNK; ++i) { ptx::mbar_init(&k_full[i], 1); ptx::mbar_init(&k_empty[i], 1); }
        for (int i = 0; i < kNV; ++i) { ptx::mbar_init(&v_full[i], 1); ptx::mbar_init(&v_empty[i], 1); }
        for (int i = 0; i < 2; ++i) {
            ptx::mbar_init(&s_full[i], 1);
            ptx::mbar_init(&p_full[i], 4);
            ptx::mbar_init(&o_bar[i], 1);
        }
        ptx::fence_mbar_init();
    }
    if (warp == 9) {
        ptx::tmem_alloc(slot, kTmemCols);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *slot;
    if (warp >= 8) {
    // ==================================================================== producer warpgroup
    ptx::setmaxnreg_dec<kProducerRegs>();
    if (warp == 8 || warp == 10) {
        // ================================================================ producers
        // warp 8: Q (both tiles), then the K ring; warp 10: the V ring.
        const bool is_k = warp == 8;
        const int NS = is_k ? kNK : kNV;
        uint64_t* full = is_k ? k_full : v_full;
        uint64_t* empty = is_k ? k_empty : v_empty;
        const CUtensorMap* map = is_k ? &tmK : &tmV;
        const int ring_off = is_k ? L::kK : L::kV;
        const int32_t* bt = a.dense ? nullptr : p.block_table + (int64_t)b * p.bt_stride;
        const int ps = a.page_size, bxt = a.box_tokens, nbox = 128 / bxt;
        const int kv_pages = a.dense ? 0 : (kv_len + ps - 1) / ps;
        const uint64_t pol = ptx::policy_evict_last();
        if (lane == 0 && n_tiles > 0) {
            ptx::prefetch_tensormap(map);
            if (is_k) {
                ptx::prefetch_tensormap(&tmQ);
                ptx::mbar_arrive_expect_tx(q_full, (uint32_t)(2 * L::kTile));
                for (int qt = 0; qt < 2; ++qt)
                    for (int dh = 0; dh < 2; ++dh) {
                        uint8_t* dst = smem + L::kQ + qt * L::kTile + dh * L::kHalf;
                        const int r0 = row0 + qt * 128;
                        if (a.q_mode == 0)
                            ptx::tma_load_5d(dst, &tmQ, q_full, 0, 0, b * p.Nq + r0 / G, dh, hk);
                        else
                            ptx::tma_load_5d(dst, &tmQ, q_full, 0, r0, dh, hk, b);
                    }
            }
        }
        int ids_reg = -1, ids_base = -(1 << 30);
        int nxt_reg = -1, nxt_base = -(1 << 30);
        auto load_ids = [&](int base) -> int {
            const int pi = base + lane;
            int id = -1;
            if (pi < kv_pages) {
                id = __ldg(bt + pi);
                if (id < 0 || id >= p.num_pages) {
                    if (is_k) record_status(p.status, KESSIE_DEV_BAD_PAGE_ID);
                    id = -1;
                }
            }
            return id;
        };
        int issued = 0;
        for (int it = 0; it < n_tiles; ++it) {
            const int key0 = (tile_lo + it) * 128;
            // page ids of this tile (at most 8 pages) from a 32-page window; the
            // next window is loaded one window ahead
            if (!a.dense) {
                const int pg_first = key0 / ps, pg_last = (key0 + 127) / ps;
                if (pg_first < ids_base || pg_last >= ids_base + 32) {
                    if (nxt_base == pg_first) { ids_base = nxt_base; ids_reg = nxt_reg; }
                    else { ids_base = pg_first; ids_reg = load_ids(ids_base); }
                    nxt_base = ids_base + 32;
                    nxt_reg = load_ids(nxt_base);
                }
            }
            int pages[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int key = key0 + u * bxt;
                const int pi = a.dense ? 0 : key / ps;
                int id = __shfl_sync(0xffffffffu, ids_reg, (pi - ids_base) & 31);
                pages[u] = (u < nbox) ? id : -1;
            }
            int ok = 1;
            if (lane == 0) {
                const int st = it % NS;
                if (it >= NS && !ptx::mbar_wait(&empty[st], ((uint32_t)(it / NS) & 1u) ^ 1u)) {
                    ok = 0;
                    record_status(p.status, KESSIE_DEV_WAIT_TIMEOUT);
                } else {
                    ptx::mbar_arrive_expect_tx(&full[st], (uint32_t)L::kTile);
                    uint8_t* dst = smem + ring_off + st * L::kTile;
                    for (int u = 0; u < nbox; ++u) {
                        const int key = key0 + u * bxt;
                        const int c1 = a.dense ? key : key % ps;
                        const int c4 = a.dense ? b : (pages[u] < 0 ? p.num_pages : pages[u]);
                        for (int dh = 0; dh < 2; ++dh)
                            ptx::tma_load_5d_hint(dst + dh * L::kHalf + u * bxt * 128, map, &full[st], 0, c1, dh, hk, c4, pol);
                    }
                    issued = it + 1;
                }
            }
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
        }
        if (lane == 0) {
            // drain: every issued load has landed before the CTA can exit
            for (int it = max(0, issued - NS); it < issued; ++it)
                if (!ptx::mbar_wait(&full[it % NS], (uint32_t)(it / NS) & 1u)) break;
        }
    } else if (warp == 9) {
        // ================================================================ MMA issuer
        // S_A(0) S_B(0) | per tile t: [P_A(t)] PV_A(t) S_A(t+1) | [P_B(t)] PV_B(t) S_B(t+1)
        // One thread issues everything, in order: S_X(t+1) overwrites the S/P
        // region X only after PV_X(t) has consumed P_X(t), and the commit that
        // publishes S_X(t+1) also covers PV_X(t).
        const uint32_t idS = ptx::umma_idesc_f16(BF16, false, 128);
        const uint32_t idPV = ptx::umma_idesc_f16(BF16, true, 128);
        const uint32_t qa = ptx::smem_u32(smem + L::kQ);
        // every wait result below is made warp-uniform (__all_sync) before it
        // steers control flow: the issue lambdas end in __syncwarp
        bool ok = n_tiles > 0 && __all_sync(0xffffffffu, ptx::mbar_wait(q_full, 0));
        ptx::tc_fence_after();
        auto issue_s = [&](int t, int x) {
            const uint32_t kb = ptx::smem_u32(smem + L::kK + (t % kNK) * L::kTile);
            const uint32_t qx = qa + (uint32_t)(x * L::kTile);
            const uint32_t dS = tmem + (uint32_t)(x * 128);
            if (lane == 0) {
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint32_t off = (uint32_t)((kk >> 2) * L::kHalf + (kk & 3) * 32);
                    ptx::umma_ss(dS, ptx::smem_desc_sw128(qx + off, 16, 1024), ptx::smem_desc_sw128(kb + off, 16, 1024),
                                 idS, kk > 0 ? 1u : 0u);
                }
                ptx::umma_commit(&s_full[x]);
                if (x == 1) ptx::umma_commit(&k_empty[t % kNK]);
            }
            __syncwarp();
        };
        auto issue_pv = [&](int t, int x) {
            const uint32_t vb = ptx::smem_u32(smem + L::kV + (t % kNV) * L::kTile);
            const uint32_t aP = tmem + (uint32_t)(x * 128);
            const uint32_t dO = tmem + 256 + (uint32_t)(x * 128);
            if (lane == 0) {
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    ptx::umma_ts(dO, aP + kk * 8, ptx::smem_desc_sw128(vb + kk * 2048, L::kHalf, 1024), idPV,
                                 (t > 0 || kk > 0) ? 1u : 0u);
                ptx::umma_commit(&o_bar[x]);
                if (x == 1) ptx::umma_commit(&v_empty[t % kNV]);
            }
            __syncwarp();
        };
        if (ok) {
            ok = __all_sync(0xffffffffu, ptx::mbar_wait(&k_full[0], 0));
            ptx::tc_fence_after();
            if (ok) { issue_s(0, 0); issue_s(0, 1); }
        }
        for (int t = 0; ok && t < n_tiles; ++t) {
            const bool more = t + 1 < n_tiles;
            if (!__all_sync(0xffffffffu, ptx::mbar_wait(&v_full[t % kNV], (uint32_t)(t / kNV) & 1u))) { ok = false; break; }
            if (!a.dense && (tile_lo + t) * 128 + 128 > kv_len) {
                // stale slots past kv_len in the last page: zero their V rows so
                // 0 * (stale NaN) cannot reach O
                uint8_t* vt = smem + L::kV + (t % kNV) * L::kTile;
                const int first = max(0, kv_len - (tile_lo + t) * 128);
                for (int e = lane; e < (128 - first) * 2 * 8; e += 32) {
                    const int row = first + e / 16, dh = (e >> 3) & 1, ch = e & 7;
                    *reinterpret_cast<uint4*>(vt + dh * L::kHalf + row * 128 + ch * 16) = make_uint4(0, 0, 0, 0);
                }
                ptx::fence_proxy_async_smem();
                __syncwarp();
            }
            if (more && !__all_sync(0xffffffffu, ptx::mbar_wait(&k_full[(t + 1) % kNK], (uint32_t)((t + 1) / kNK) & 1u))) {
                ok = false;
                break;
            }
            for (int x = 0; x < 2; ++x) {
                if (!__all_sync(0xffffffffu, ptx::mbar_wait(&p_full[x], (uint32_t)t & 1u))) { ok = false; break; }
                ptx::tc_fence_after();
                issue_pv(t, x);
                if (more) issue_s(t + 1, x);
            }
        }
        if (!ok && n_tiles > 0) record_status(p.status, KESSIE_DEV_WAIT_TIMEOUT);
    }
    } else {
        // ================================================================ softmax warpgroups
        ptx::setmaxnreg_inc<kSoftmaxRegs>();
        const int x = warp >> 2;                       // Q tile: 0 (warps 0-3) or 1 (warps 4-7)
        const int q4 = warp & 3;
        const int r = q4 * 32 + lane;
        const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
        const uint32_t sreg = tmem + lane_off + (uint32_t)(x * 128);
        const uint32_t oreg = tmem + lane_off + 256 + (uint32_t)(x * 128);
        const int rr = row0 + x * 128 + r;
        const bool valid_row = rr < rows_total;
        const int tok = rr / G, gh = rr - tok * G;
        const int pos = q0 + tok;
        // this Q tile's position range (interior-tile test)
        const int xr0 = min(row0 + x * 128, rows_total - 1), xr1 = min(row0 + x * 128 + 127, rows_total - 1);
        const int xpos_lo = q0 + xr0 / G, xpos_hi = q0 + xr1 / G;
        int hi_r = min(kv_len, (p.causal || p.window > 0) ? pos + 1 : kv_len);
        int lo_r = p.window > 0 ? pos - p.window + 1 : 0;
        if (!valid_row) hi_r = lo_r - 1;
        float m_used = -INFINITY, l = 0.f;
        bool ok = true;
        float* wbuf = reinterpret_cast<float*>(smem + L::kW) + warp * 128;
        float* bbuf = reinterpret_cast<float*>(smem + L::kB) + warp * 128;
        const bool has_bias = p.bias.on != 0;
        const int bias_fb = has_bias ? fog_bias_boundary(p.bias, kv_len) : 0;
        // the bias enters as raw-score units (bias / sm_scale) so the exponent
        // s * scale * log2e below adds exactly bias * log2e
        const float bias_to_raw = has_bias ? kLog2eTc / p.scale_log2 : 0.f;
        const float inv_den = 1.f / (float)max(cs - 1, 1);
        for (int j = 0; j < n_tiles; ++j) {
            const int key0 = (tile_lo + j) * 128;
            if (has_fog) {
                // this warp's copy of the tile's fog weights (kessie_hip_kernels.py:411-412):
                // (key / (cs-1))^alpha as 2^(alpha * log2(key / (cs-1))) on the MUFU
                float4 w4v;
                float* w = &w4v.x;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int key = key0 + lane * 4 + e;
                    float wv;
                    if (key >= kv_len) wv = 0.f;
                    else if (p.fog_w) wv = __ldg(p.fog_w + b * p.fog_w_sb + key);
                    else if (key >= cs) wv = 1.f;
                    else wv = ptx::ex2(p.fog_alpha * ptx::lg2((float)key * inv_den));
                    w[e] = wv;
                }
                reinterpret_cast<float4*>(wbuf)[lane] = w4v;
            }
            if (has_bias) {
                float4 b4v;
                float* bq = &b4v.x;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int key = key0 + lane * 4 + e;
                    bq[e] = key < kv_len ? fog_bias_at(p.bias, bias_fb, key) * bias_to_raw : 0.f;
                }
                reinterpret_cast<float4*>(bbuf)[lane] = b4v;
            }
            __syncwarp();
            // warp-uniform: the tcgen05.ld / st below are warp-collective
            if (!__all_sync(0xffffffffu, ptx::mbar_wait(&s_full[x], (uint32_t)j & 1u))) { ok = false; break; }
            ptx::tc_fence_after();
            uint32_t sv[4][32];
#pragma unroll
            for (int c = 0; c < 4; ++c) ptx::tmem_ld32(sreg + c * 32, sv[c]);
            ptx::tmem_ld_wait();
            const bool interior = !has_bias && key0 + 128 <= kv_len &&
                                  (!(p.causal || p.window > 0) || key0 + 127 <= xpos_lo) &&
                                  (p.window <= 0 || key0 >= xpos_hi - p.window + 1);
            float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
            if (interior && valid_row) {
#pragma unroll
                for (int c = 0; c < 4; ++c)
#pragma unroll
                    for (int i = 0; i < 32; i += 2)
                        mx4[(i >> 1) & 3] = ptx::max3(mx4[(i >> 1) & 3], __uint_as_float(sv[c][i]),
                                                      __uint_as_float(sv[c][i + 1]));
            } else {
#pragma unroll
                for (int c = 0; c < 4; ++c)
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const int key = key0 + c * 32 + i;
                        const float sb = has_bias ? bbuf[c * 32 + i] : 0.f;
                        const float sx = (key >= lo_r && key < hi_r) ? __uint_as_float(sv[c][i]) + sb : -INFINITY;
                        sv[c][i] = __float_as_uint(sx);
                        mx4[i & 3] = fmaxf(mx4[i & 3], sx);
                    }
            }
            const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
            const float m_tile = mx == -INFINITY ? -INFINITY : mx * p.scale_log2;
            const float m_new = fmaxf(m_used, m_tile);
            const bool need = m_new != -INFINITY && (m_used == -INFINITY || m_new > m_used + kRescaleThreshold);
            float factor = 1.f;
            if (need) {
                factor = m_used == -INFINITY ? 0.f : ptx::ex2(m_used - m_new);
                l *= factor;
                m_used = m_new;
            }
            const float nb = m_used == -INFINITY ? 0.f : -m_used;
            l += has_fog ? softmax_p_tile<BF16, true>(sv, sreg, p.scale_log2, nb, wbuf)
                         : softmax_p_tile<BF16, false>(sv, sreg, p.scale_log2, nb, wbuf);
            // O rescale in TMEM (warp-collective, rare), after P so the scores'
            // registers are free.  PV(j-1) is complete (the commit that
            // published S(j) was issued after it) and PV(j) waits for p_full.
            if (__any_sync(0xffffffffu, need && factor != 0.f && j > 0)) {
                const float f = (need && factor != 0.f) ? factor : 1.f;
#pragma unroll 1
                for (int c = 0; c < 4; ++c) {
                    uint32_t ov[32];
                    ptx::tmem_ld32(oreg + c * 32, ov);
                    ptx::tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * f);
                    ptx::tmem_st32(oreg + c * 32, ov);
                }
                ptx::tmem_st_wait();
            }
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&p_full[x]);
        }
        // ---- epilogue: O / l -> global
        bool have = n_tiles > 0 && ok;
        if (have) {
            have = __all_sync(0xffffffffu, ptx::mbar_wait(&o_bar[x], (uint32_t)(n_tiles - 1) & 1u));
            ptx::tc_fence_after();
        }
        if (!ok || (n_tiles > 0 && !have)) record_status(p.status, KESSIE_DEV_WAIT_TIMEOUT);
        const float inv = l > 0.f ? 1.f / l : 0.f;
        uint16_t* orow = reinterpret_cast<uint16_t*>(p.o) + (int64_t)b * p.o_sb + (int64_t)tok * p.o_st +
                         (int64_t)(hk * G + gh) * p.o_sh;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
            uint32_t ov[32];
            if (have) {
                ptx::tmem_ld32(oreg + c * 32, ov);
                ptx::tmem_ld_wait();
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) ov[i] = 0u;
            }
            if (valid_row) {
                uint32_t pk[16];
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    pk[i] = ptx::pack2<BF16>(__uint_as_float(ov[2 * i]) * inv, __uint_as_float(ov[2 * i + 1]) * inv);
                uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
                for (int v = 0; v < 4; ++v) dst[v] = make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
            }
        }
    }
    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace

int run_prefill_tc(const PrefillParams& p, const void* q_base, const void* k_cache, const void* v_cache,
                   int64_t page_stride, int64_t token_stride, int64_t head_stride, int map_pages, int map_tokens,
                   int head_dim, bool bf16, cudaStream_t st) {
    const char* env = getenv("KESSIE_PREFILL_IMPL");
    if (env && strcmp(env, "mma") == 0) return kTcNotCovered;
    if (head_dim != 128 || p.G <= 0 || 128 % p.G) return kTcNotCovered;
    // alignment: Q/O rows and K/V rows 16-byte aligned
    if (((p.q_st | p.q_sh | p.o_st | p.o_sh) & 7) || ((token_stride | head_stride | page_stride) & 7))
        return kTcNotCovered;
    const bool dense = p.block_table == nullptr;
    int q_mode;
    if (p.B == 1 || p.q_sb == (int64_t)p.Nq * p.q_st) q_mode = 0;
    else if (p.G == 1) q_mode = 1;
    else return kTcNotCovered;
    const int ps = map_tokens;
    int box = dense ? 128 : (ps >= 128 ? 128 : ps);
    if (!dense && (ps % 16 || 128 % box)) return kTcNotCovered;

    CUtensorMap mq, mk, mv;
    CUresult r;
    if (q_mode == 0) {
        const cuuint64_t dims[5] = {64, (cuuint64_t)p.G, (cuuint64_t)p.B * p.Nq, 2, (cuuint64_t)p.Hkv};
        const cuuint64_t str[4] = {(cuuint64_t)p.q_sh * 2, (cuuint64_t)p.q_st * 2, 128, (cuuint64_t)p.G * p.q_sh * 2};
        const cuuint32_t bx[5] = {64, (cuuint32_t)p.G, (cuuint32_t)(128 / p.G), 1, 1};
        r = encode_tiled_5d_sw128(&mq, q_base, bf16, dims, str, bx);
    } else {
        const cuuint64_t dims[5] = {64, (cuuint64_t)p.Nq, 2, (cuuint64_t)p.Hq, (cuuint64_t)p.B};
        const cuuint64_t str[4] = {(cuuint64_t)p.q_st * 2, 128, (cuuint64_t)p.q_sh * 2, (cuuint64_t)p.q_sb * 2};
        const cuuint32_t bx[5] = {64, 128, 1, 1, 1};
        r = encode_tiled_5d_sw128(&mq, q_base, bf16, dims, str, bx);
    }
    if (r != CUDA_SUCCESS) return kTcNotCovered;
    {
        const cuuint64_t dims[5] = {64, (cuuint64_t)map_tokens, 2, (cuuint64_t)p.Hkv, (cuuint64_t)map_pages};
        const cuuint64_t str[4] = {(cuuint64_t)token_stride * 2, 128, (cuuint64_t)head_stride * 2,
                                   (cuuint64_t)page_stride * 2};
        const cuuint32_t bx[5] = {64, (cuuint32_t)box, 1, 1, 1};
        if (encode_tiled_5d_sw128(&mk, k_cache, bf16, dims, str, bx) != CUDA_SUCCESS ||
            encode_tiled_5d_sw128(&mv, v_cache, bf16, dims, str, bx) != CUDA_SUCCESS)
            return kTcNotCovered;
    }
    TcArgs a;
    a.p = p;
    a.q_mode = q_mode;
    a.box_tokens = box;
    a.dense = dense ? 1 : 0;
    a.page_size = ps;
    auto kern = bf16 ? fog_prefill_tc_kernel<true> : fog_prefill_tc_kernel<false>;
    // setmaxnreg.inc waits until the CTA's register pool can satisfy it, so the
    // split is only valid if the kernel was built with kLaunchRegs per thread.
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess) { cudaGetLastError(); return kTcNotCovered; }
    if (fa.numRegs < kLaunchRegs) return kTcNotCovered;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc) != cudaSuccess)
        return check_launch("prefill_tc: set smem attribute");
    const int rows = p.Nq * p.G;
    dim3 grid((rows + kRowsPerCta - 1) / kRowsPerCta, p.Hkv, p.B);
    kern<<<grid, kThreads, L::kAlloc, st>>>(mq, mk, mv, a);
    return check_launch("fog_prefill_tc");
}

}  // namespace kessie
