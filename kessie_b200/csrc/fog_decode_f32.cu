// fog_decode_f32.cu -- paged fog-attention decode in fp32 on the CUDA cores.
//
// Semantics are those of the bf16/fp16 decode (fog_decode.cu) and of the
// reference's fp32 path, kessie_fused_fog_attention_ref
// (kessie_hip_kernels.py:577-593) at one query row per sequence:
//     O = sum_j p_j w_j v_j / sum_j p_j,  p_j = exp(q.k_j * sm_scale - m),
// over the visible keys (j <= q_pos; q_pos - j < W when W > 0), with the fog
// weight w_j = (j / max(cs-1, 1))^alpha for j < cs (kessie_hip_kernels.py:408-412)
// evaluated with an IEEE divide and powf (sqrtf for alpha 0.5), as the
// reference's fp32 torch ops do.  Every product and sum is fp32; no tensor
// core is involved (tf32 would miss the 1e-4 fp32 bar).
//
// Design (B200): decode reads 1 KB of K+V per key (D 128) and does 4 FLOP per
// byte, so it is HBM-bound as long as the FMA work per key stays below the
// issue budget.
//   grid  = (S splits, B*Hkv groups); the visible keys of a group are cut into
//           8-key chunks (a chunk never crosses a page: page_size % 16 == 0)
//           and split S ways; S is chosen from the SM count so the grid's
//           last wave is nearly full (one wave when one fills nearly as
//           well), with at least two chunks per warp.
//   CTA   = 8 warps.  Each warp streams every 8th chunk of the CTA's range
//           through its own 3-stage ring: per chunk two TMA box loads (K, V;
//           8 keys x D of one head, 4 KB each at D 128) on the stage's
//           mbarrier, so two chunks per warp are in flight while it computes
//           the third.  Page ids come from the block table 32 chunks at a
//           time, a batch ahead, one per lane.  The boxes land 128-byte
//           swizzled (16-byte chunk c of key t at row (c/8)*8 + t, position
//           (c%8) ^ t), which both the score and the PV reads take without
//           bank conflicts.
//   QK    = lane (key kk = lane/4, quarter dq = lane%4) dots its quarter row of
//           K with every query head of the group, two heads per packed fp32
//           FMA (fma.rn.f32x2; q staged once per CTA by head pairs, pre-scaled
//           by sm_scale*log2e, swizzled so the four quarters read distinct
//           banks, and at GP 4 held in registers for the whole range); a
//           two-step transposing shuffle reduction over the
//           quarters leaves each lane the full scores of GP/4 heads of its key.
//   soft  = online softmax per head across the chunk's 8 keys with a lazy
//           max: the running max m moves (xor-shuffle max over the key lanes,
//           rescale of l and O) only when a score passes it by more than
//           kSlack = 8 (log2 units), so p <= 2^8 and most chunks need no
//           reduction; each key lane keeps its share of l and its true max,
//           summed / reduced once at the end, where (m, l, O) move to the
//           true max so the merges and the partials carry it.  p*w and the
//           rescale factors go to a per-warp shared tile.
//   PV    = lane owns D/32 consecutive dims of O for every head; per key one
//           V load and GP*D/64 packed FMAs (two heads each), with no per-key
//           branch: masked keys of a partial chunk have their V rows zeroed.
//   What bounds it is the per-warp dependency chain per chunk (8 warps per
//   SM; fewer warps with deeper rings measured slower), so the loop keeps
//   shuffles, votes and branches off the common path.
//   merge = the 8 warps merge through shared memory; with S > 1 each CTA
//           writes (O/l, m, l) per head into its workspace slot and bumps the
//           group's tagged arrival counter; the last CTA merges the S slots
//           and writes out / out_partial (and zeroes the counter).
#include "decode_f32.cuh"
#include "ptx.cuh"
#include "tma_host.cuh"

#include <math.h>

namespace kessie {
namespace {

constexpr int kW = 8;            // warps per CTA
constexpr int kT = kW * 32;
constexpr int kNS = 3;           // shared-memory stages per warp
constexpr float kSlack = 8.f;    // log2 units a score may pass the running max by before it moves
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr unsigned kFull = 0xffffffffu;

// Shared memory (floats, from a 1024-byte aligned base): the warps' stage
// rings first (every stage and tile 1024-byte aligned, as the 128-byte
// swizzle needs), then q, the per-warp P / alpha tiles, the merge tail and the
// per-warp mbarriers.
template <int D, int GP>
struct F32Layout {
    static constexpr int kChunk = 8 * D;                     // floats of one 8-key K (or V) tile
    static constexpr int kStage = 2 * kChunk;
    static constexpr int kRing = kNS * kStage;               // one warp's stages
    static constexpr int kQOff = kW * kRing;                 // staged q [GP][D]
    static constexpr int kWarpOff = kQOff + GP * D;          // per warp: P tile [8][GP], alpha [GP]
    static constexpr int kWarpF = 8 * GP + GP;
    static constexpr int kTailOff = kWarpOff + kW * kWarpF;  // merged (M, L) [GP][2], warp scales [kW][GP]
    static constexpr int kBarOff = (kTailOff + 2 * GP + kW * GP + 1) & ~1;   // kW x kNS mbarriers
    static constexpr int kFloats = kBarOff + 2 * kW * kNS;
    static constexpr int kBytes = kFloats * 4 + 1024;        // + slack to align the dynamic base
    static_assert(kRing >= 2 * GP + GP * D, "a warp's merge data must fit in its stages");
    static_assert((kChunk * 4) % 1024 == 0, "tiles must stay 1024-byte aligned");
    static_assert(kWarpF % 4 == 0 && kWarpOff % 4 == 0, "float4 alignment");
};

// Offset (floats) of dims [4c, 4c + 4) of key t (0..7) in an 8-key tile: row
// (c / 8) * 8 + t of 32 floats, 16-byte chunk c % 8 XOR t -- the layout a
// 128-byte swizzled TMA box {32, 8 tokens, D/32} lands in.
__device__ __forceinline__ int tile_off(int t, int c) { return ((c >> 3) * 8 + t) * 32 + (((c & 7) ^ t) << 2); }

struct SeqF32 {
    int k_lo, k_hi;   // visible local keys [k_lo, k_hi)
    int off;          // global position of local key 0
    int cs;           // clear_start (global), 0: no fog
};

__device__ __forceinline__ SeqF32 seq_f32(const DecodeF32Args& p, int b) {
    SeqF32 s;
    if (p.square_n > 0) {
        const int qp = (p.causal || p.window > 0) ? p.square_row0 + b : p.square_n - 1;
        s.off = 0;
        s.k_hi = min(p.square_n, qp + 1);
        s.k_lo = p.window > 0 ? max(0, qp - p.window + 1) : 0;
        if (s.k_hi < s.k_lo) s.k_hi = s.k_lo;
        s.cs = 0;
        return s;
    }
    const int cap = ((p.max_seq_len + 15) / 16) * 16;
    int n = p.seq_lens[b];
    if (n < 0 || n > cap) {
        record_status(p.status, KESSIE_DEV_BAD_ARG);
        n = n < 0 ? 0 : cap;
    }
    s.off = p.kv_off ? p.kv_off[b] : 0;
    const int qp = p.q_pos ? p.q_pos[b] : s.off + n - 1;
    s.k_hi = min(n, qp - s.off + 1);
    s.k_lo = p.window > 0 ? max(0, qp - p.window + 1 - s.off) : 0;
    if (s.k_hi < s.k_lo) s.k_hi = s.k_lo;
    s.cs = p.clear_start ? p.clear_start[b] : 0;
    return s;
}

// Fog weight of the key at global position j (kessie_hip_kernels.py:408-412):
// the fp32 ratio j / max(cs-1, 1) with an IEEE divide, then pow (sqrt for
// alpha 0.5, the route torch takes for that exponent).
__device__ __forceinline__ float fog_weight_f32(const DecodeF32Args& p, int cs, int j) {
    if (p.fog_w) return __ldg(p.fog_w + j);
    if (!(p.fog_alpha > 0.f) || cs <= 0 || j >= cs) return 1.f;
    const float t = __fdiv_rn((float)j, (float)max(cs - 1, 1));
    return p.fog_alpha == 0.5f ? sqrtf(t) : powf(t, p.fog_alpha);
}

// Count one arrival at a group counter; returns the arrivals before this one
// (a counter holding another launch's tag counts as zero).
__device__ __forceinline__ unsigned arrive_tagged(unsigned long long* c, uint32_t tag) {
    const unsigned long long hi = (unsigned long long)tag << 32;
    unsigned long long old = *reinterpret_cast<volatile unsigned long long*>(c);
    while (true) {
        const unsigned long long cur = (old >> 32) == tag ? old : hi;
        const unsigned long long prev = atomicCAS(c, old, cur + 1ull);
        if (prev == old) return (unsigned)(cur & 0xffffffffull);
        old = prev;
    }
}

__device__ __forceinline__ void emit_f32(const DecodeF32Args& p, int b, int h, int d, float o, float M, float L) {
    const int D = p.D;
    if (p.out) p.out[(int64_t)b * p.out_sb + (int64_t)h * p.out_sh + d] = o;
    if (p.out_part) {
        float* dst = p.out_part + ((int64_t)b * p.Hq + h) * (D + 2);
        dst[d] = o;
        if (d == 0) {
            dst[D] = M == -INFINITY ? -INFINITY : M * kLn2;
            dst[D + 1] = L;
        }
    }
}

template <int D, int GP>
__global__ void __launch_bounds__(kT, 1) fog_decode_f32_kernel(const DecodeF32Args p, const int S,
                                                               const __grid_constant__ CUtensorMap tmK,
                                                               const __grid_constant__ CUtensorMap tmV,
                                                               const int dense) {
    using Lay = F32Layout<D, GP>;
    constexpr int E = D / 32;      // PV: consecutive dims of O per lane
    constexpr int CPL = D / 16;    // QK: 16-byte chunks per lane (a quarter row)
    constexpr int H4 = GP / 4;     // QK: heads per lane after the reduction
    extern __shared__ float4 smem_f4[];
    float* sm = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(smem_f4) + 1023) & ~uintptr_t(1023));
    float* sq = sm + Lay::kQOff;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* sw = sm + warp * Lay::kRing;
    float* sP = sm + Lay::kWarpOff + warp * Lay::kWarpF;
    float* sA = sP + 8 * GP;
    float* sML = sm + Lay::kTailOff;       // [GP][2]
    float* sSC = sML + 2 * GP;             // [kW][GP]
    __shared__ int s_last;

    const int grp = blockIdx.y, split = blockIdx.x;
    const int b = grp / p.Hkv, hk = grp - b * p.Hkv;
    const int G = p.Hq / p.Hkv;
    const SeqF32 si = seq_f32(p, b);

    // query rows of the group, scaled into log2 units, stored by head pairs:
    // 16-byte chunk c of pair gp holds dims 2c, 2c+1 of heads 2gp, 2gp+1
    // ([q(2gp,2c), q(2gp+1,2c), q(2gp,2c+1), q(2gp+1,2c+1)]), the chunk index
    // XORed with its quarter so the four quarters read distinct banks
    const float qscale = p.sm_scale * kLog2e;
    constexpr int QC = D / 8;                  // chunks per quarter of a head pair's row
    for (int i = threadIdx.x; i < GP * D; i += kT) {
        const int g = i / D, d = i - g * D;
        float v = 0.f;
        if (g < G) v = p.q[(int64_t)b * p.q_sb + (int64_t)(hk * G + g) * p.q_sh + d] * qscale;
        const int c = d >> 1, dq = c / QC;
        sq[((g >> 1) * (D / 2) + (c ^ dq)) * 4 + (d & 1) * 2 + (g & 1)] = v;
    }
    __syncthreads();

    // this CTA's chunks: [cb, ce) of the group's visible chunks
    const int c_lo = si.k_lo >> 3;
    const int nch = si.k_hi > si.k_lo ? ((si.k_hi + 7) >> 3) - c_lo : 0;
    const int per = (nch + S - 1) / S;
    const int cb = c_lo + split * per;
    const int ce = min(c_lo + nch, cb + per);
    const int nw = ce > cb + warp ? (ce - cb - warp + kW - 1) / kW : 0;
    const int32_t* bt = p.block_table ? p.block_table + (int64_t)b * p.bt_stride : nullptr;

    // Page ids come from the block table 32 chunks at a time, a batch ahead:
    // lane j holds the page of this warp's chunk 32 * batch + j, so a copy
    // never waits on a block-table load.
    auto page_of = [&](int i) -> int {
        if (i >= nw) return 0;
        const int pi = (cb + warp + i * kW) * 8 / p.page_size;
        return bt ? __ldg(bt + pi) : pi;
    };
    int pg_cur = page_of(lane), pg_next = page_of(32 + lane);

    // Per warp one mbarrier per stage.
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + Lay::kBarOff) + warp * kNS;
    if (lane == 0) {
#pragma unroll
        for (int s2 = 0; s2 < kNS; ++s2) ptx::mbar_init(&bars[s2], 1);
        ptx::fence_mbar_init();
        ptx::prefetch_tensormap(&tmK);
        ptx::prefetch_tensormap(&tmV);
    }
    __syncwarp();

    // Starts the two box loads (K, V; 8 keys x D each) of this warp's chunk i
    // into stage i % kNS on the stage's mbarrier (chunks are issued in
    // increasing order); returns true (and copies nothing, the barrier
    // completing at once) when the chunk's page id is out of range.  Rows past
    // the visible end are in-page (zero-filled past a dense cache's end) and
    // masked.
    auto issue = [&](int i) -> bool {
        if ((i & 31) == 0 && i > 0) {
            pg_cur = pg_next;
            pg_next = page_of(i + 32 + lane);
        }
        const int key0 = (cb + warp + i * kW) * 8;
        const int pi = key0 / p.page_size, tok = key0 - pi * p.page_size;
        const int page = __shfl_sync(kFull, pg_cur, i & 31);
        uint64_t* bar = &bars[i % kNS];
        if (page < 0 || page >= p.num_pages) {
            if (lane == 0) {
                record_status(p.status, KESSIE_DEV_BAD_PAGE_ID);
                ptx::mbar_arrive(bar);
            }
            return true;
        }
        if (lane == 0) {
            float* dK = sw + (i % kNS) * Lay::kStage;
            float* dV = dK + Lay::kChunk;
            ptx::mbar_arrive_expect_tx(bar, (uint32_t)(2 * Lay::kChunk * 4));
            if (dense) {
                ptx::tma_load_4d(dK, &tmK, bar, 0, key0, 0, hk);
                ptx::tma_load_4d(dV, &tmV, bar, 0, key0, 0, hk);
            } else {
                ptx::tma_load_5d(dK, &tmK, bar, 0, tok, 0, hk, page);
                ptx::tma_load_5d(dV, &tmV, bar, 0, tok, 0, hk, page);
            }
        }
        return false;
    };

    float m[H4], l[H4], mx[H4];     // running (m, l) of the heads; mx: this key lane's true max
#pragma unroll
    for (int h = 0; h < H4; ++h) { m[h] = -INFINITY; l[h] = 0.f; mx[h] = -INFINITY; }
    uint64_t acc2[GP / 2][E];       // (acc[2gp][e], acc[2gp+1][e]) as packed fp32 pairs
#pragma unroll
    for (int gp = 0; gp < GP / 2; ++gp)
#pragma unroll
        for (int e = 0; e < E; ++e) acc2[gp][e] = 0ull;

    uint32_t badm = 0;   // bit s: the chunk in stage s had a bad page id (warp-uniform)
#pragma unroll
    for (int i = 0; i < kNS - 1; ++i) {
        if (i < nw) {
            if (issue(i)) badm |= 1u << i; else badm &= ~(1u << i);
        }
        cp_async_commit();
    }
    const int kk = lane >> 2, dq = lane & 3;
    // At GP 4 the lane's q slice (its quarter of 4 heads: 128 floats) stays in
    // registers for the whole range, halving the shared loads per chunk; at
    // GP 8 / 16 it does not fit, and the loop reads it from shared memory.
    constexpr bool kQReg = GP == 4;
    constexpr int kQG = kQReg ? GP / 2 : 1, kQC = kQReg ? CPL : 1;
    float4 qreg[kQG][kQC][2];
    if (kQReg) {
#pragma unroll
        for (int gp = 0; gp < kQG; ++gp)
#pragma unroll
            for (int cc = 0; cc < kQC; ++cc) {
                const int c0 = dq * QC + 2 * cc;
                qreg[gp][cc][0] = *reinterpret_cast<const float4*>(sq + (gp * (D / 2) + (c0 ^ dq)) * 4);
                qreg[gp][cc][1] = *reinterpret_cast<const float4*>(sq + (gp * (D / 2) + ((c0 + 1) ^ dq)) * 4);
            }
    }
    int stuck = -1;      // chunk whose wait gave up (warp-uniform); the rest is not read
    for (int i = 0; i < nw; ++i) {
        const bool ok = __all_sync(kFull, ptx::mbar_wait(&bars[i % kNS], (uint32_t)(i / kNS) & 1u));
        __syncwarp();                      // every lane is done with the stage refilled next
        if (!ok) {
            if (lane == 0) record_status(p.status, KESSIE_DEV_WAIT_TIMEOUT);
            stuck = i;
            break;
        }
        {
            const int nx = i + kNS - 1;
            if (nx < nw) {
                const int sl = nx % kNS;
                if (issue(nx)) badm |= 1u << sl; else badm &= ~(1u << sl);
            }
            cp_async_commit();
        }
        const int sl = i % kNS;
        const float* sK = sw + sl * Lay::kStage;
        const float* sV = sK + Lay::kChunk;
        const bool bad = (badm >> sl) & 1u;
        const int key0 = (cb + warp + i * kW) * 8;

        // ---- scores: lane (kk, dq) dots its quarter of key kk with every head,
        // two heads per packed fma (fma.rn.f32x2)
        uint64_t s2[GP / 2];
#pragma unroll
        for (int gp = 0; gp < GP / 2; ++gp) s2[gp] = 0ull;
#pragma unroll
        for (int cc = 0; cc < CPL; ++cc) {
            const int x = dq * CPL + cc;
            const float4 kf = *reinterpret_cast<const float4*>(sK + tile_off(kk, x));
            const uint64_t kx = ptx::f2_pack(kf.x, kf.x), ky = ptx::f2_pack(kf.y, kf.y);
            const uint64_t kz = ptx::f2_pack(kf.z, kf.z), kw = ptx::f2_pack(kf.w, kf.w);
            const int c0 = dq * QC + 2 * cc;           // chunks of dims 4cc.. 4cc+3 of the quarter
#pragma unroll
            for (int gp = 0; gp < GP / 2; ++gp) {
                const float4 qa = kQReg ? qreg[kQReg ? gp : 0][kQReg ? cc : 0][0]
                                        : *reinterpret_cast<const float4*>(sq + (gp * (D / 2) + (c0 ^ dq)) * 4);
                const float4 qb = kQReg ? qreg[kQReg ? gp : 0][kQReg ? cc : 0][1]
                                        : *reinterpret_cast<const float4*>(sq + (gp * (D / 2) + ((c0 + 1) ^ dq)) * 4);
                s2[gp] = ptx::ffma2(ptx::f2_pack(qa.x, qa.y), kx, s2[gp]);
                s2[gp] = ptx::ffma2(ptx::f2_pack(qa.z, qa.w), ky, s2[gp]);
                s2[gp] = ptx::ffma2(ptx::f2_pack(qb.x, qb.y), kz, s2[gp]);
                s2[gp] = ptx::ffma2(ptx::f2_pack(qb.z, qb.w), kw, s2[gp]);
            }
        }
        float s[GP];
#pragma unroll
        for (int gp = 0; gp < GP / 2; ++gp) ptx::f2_unpack(s2[gp], s[2 * gp], s[2 * gp + 1]);
        // transposing reduction over the quarters: lane keeps heads dq*H4 .. dq*H4+H4-1
        float t[GP / 2];
        {
            const bool up = (lane & 2) != 0;
#pragma unroll
            for (int j = 0; j < GP / 2; ++j) {
                const float send = up ? s[j] : s[j + GP / 2];
                const float keep = up ? s[j + GP / 2] : s[j];
                t[j] = keep + __shfl_xor_sync(kFull, send, 2);
            }
        }
        float u[H4];
        {
            const bool up = (lane & 1) != 0;
#pragma unroll
            for (int j = 0; j < H4; ++j) {
                const float send = up ? t[j] : t[j + H4];
                const float keep = up ? t[j + H4] : t[j];
                u[j] = keep + __shfl_xor_sync(kFull, send, 1);
            }
        }

        // ---- online softmax over the chunk's 8 keys
        const int jl = key0 + kk;
        const bool valid = !bad && jl >= si.k_lo && jl < si.k_hi;
        const float w = valid ? fog_weight_f32(p, si.cs, si.off + jl) : 0.f;
        // The running max m moves only when a score passes it by more than
        // kSlack (log2 units): p = 2^(x - m) stays <= 2^kSlack, and a chunk
        // that passes no lane's bound needs no max reduction and no rescale.
        float x[H4];
        bool over = false;
#pragma unroll
        for (int h = 0; h < H4; ++h) {
            x[h] = valid ? u[h] : -INFINITY;
            over |= x[h] > m[h] + kSlack;
            mx[h] = fmaxf(mx[h], x[h]);
        }
        const bool rescale = __any_sync(kFull, over);          // warp-uniform
        if (rescale) {
#pragma unroll
            for (int h = 0; h < H4; ++h) {
                float cm = x[h];
                cm = fmaxf(cm, __shfl_xor_sync(kFull, cm, 4));
                cm = fmaxf(cm, __shfl_xor_sync(kFull, cm, 8));
                cm = fmaxf(cm, __shfl_xor_sync(kFull, cm, 16));
                const float mn = fmaxf(m[h], cm);
                const float al = mn == -INFINITY ? 1.f : exp2f(m[h] - mn);
                l[h] *= al;
                m[h] = mn;
                if (kk == 0) sA[dq * H4 + h] = al;
            }
        }
#pragma unroll
        for (int h = 0; h < H4; ++h) {
            const float pr = valid ? exp2f(x[h] - m[h]) : 0.f;
            l[h] += pr;                        // this key lane's share; summed over the key lanes at the end
            sP[kk * GP + dq * H4 + h] = pr * w;
        }
        __syncwarp();

        // ---- O += P * V (fog already in P); lane owns dims lane*E .. lane*E+E-1
        if (rescale) {
#pragma unroll
            for (int g4 = 0; g4 < GP / 4; ++g4) {
                const float4 a = *reinterpret_cast<const float4*>(sA + g4 * 4);
                const uint64_t a01 = ptx::f2_pack(a.x, a.y), a23 = ptx::f2_pack(a.z, a.w);
#pragma unroll
                for (int e = 0; e < E; ++e) {
                    acc2[g4 * 2][e] = ptx::fmul2(acc2[g4 * 2][e], a01);
                    acc2[g4 * 2 + 1][e] = ptx::fmul2(acc2[g4 * 2 + 1][e], a23);
                }
            }
        }
        // masked keys of a partial chunk (first / last of a range, or a bad
        // page) get zero V rows, so the PV loop needs no per-key branch and
        // 0 * (stale NaN) cannot reach O; each lane zeroes the dims it reads
        const bool partial = bad || key0 < si.k_lo || key0 + 8 > si.k_hi;    // warp-uniform
        if (partial) {
            float* zV = sw + sl * Lay::kStage + Lay::kChunk;
#pragma unroll
            for (int r = 0; r < 8; ++r) {
                const int j = key0 + r;
                if (!(bad || j < si.k_lo || j >= si.k_hi)) continue;
                if (E == 4) *reinterpret_cast<float4*>(zV + tile_off(r, lane)) = make_float4(0.f, 0.f, 0.f, 0.f);
                else *reinterpret_cast<float2*>(zV + tile_off(r, lane >> 1) + (lane & 1) * 2) = make_float2(0.f, 0.f);
            }
        }
#pragma unroll
        for (int r = 0; r < 8; ++r) {
            uint64_t v2[E];                                        // (v[e], v[e]): one V value for a head pair
            if (E == 4) {
                const float4 vf = *reinterpret_cast<const float4*>(sV + tile_off(r, lane));
                v2[0] = ptx::f2_pack(vf.x, vf.x); v2[1] = ptx::f2_pack(vf.y, vf.y);
                v2[2] = ptx::f2_pack(vf.z, vf.z); v2[3] = ptx::f2_pack(vf.w, vf.w);
            } else {
                const float2 vf = *reinterpret_cast<const float2*>(sV + tile_off(r, lane >> 1) + (lane & 1) * 2);
                v2[0] = ptx::f2_pack(vf.x, vf.x); v2[1] = ptx::f2_pack(vf.y, vf.y);
            }
#pragma unroll
            for (int g4 = 0; g4 < GP / 4; ++g4) {
                const float4 pq = *reinterpret_cast<const float4*>(sP + r * GP + g4 * 4);
                const uint64_t p01 = ptx::f2_pack(pq.x, pq.y), p23 = ptx::f2_pack(pq.z, pq.w);
#pragma unroll
                for (int e = 0; e < E; ++e) {
                    acc2[g4 * 2][e] = ptx::ffma2(p01, v2[e], acc2[g4 * 2][e]);
                    acc2[g4 * 2 + 1][e] = ptx::ffma2(p23, v2[e], acc2[g4 * 2 + 1][e]);
                }
            }
        }
        // the zero rows (generic proxy) are ordered before the TMA refill of
        // this stage (async proxy), which follows the next iteration's warp barrier
        if (partial) ptx::fence_proxy_async_smem();
    }
    if (stuck >= 0) {
        // box loads still in flight land before the stages are reused
        for (int j = stuck; j < min(nw, stuck + kNS - 1); ++j)
            (void)__all_sync(kFull, ptx::mbar_wait(&bars[j % kNS], (uint32_t)(j / kNS) & 1u));
    }
    __syncthreads();

    // ---- merge the 8 warps (each writes into its own stage area)
    float* mw = sw;              // [GP][2] (m, l)
    float* ow = sw + 2 * GP;     // [GP][D]
    // The running max trails the true max by at most kSlack: move the warp's
    // (m, l, O) to the true max, so the merges and the reported partials
    // carry the exact maximum.
#pragma unroll
    for (int h = 0; h < H4; ++h) {
        l[h] += __shfl_xor_sync(kFull, l[h], 4);
        l[h] += __shfl_xor_sync(kFull, l[h], 8);
        l[h] += __shfl_xor_sync(kFull, l[h], 16);
        float mt = mx[h];
        mt = fmaxf(mt, __shfl_xor_sync(kFull, mt, 4));
        mt = fmaxf(mt, __shfl_xor_sync(kFull, mt, 8));
        mt = fmaxf(mt, __shfl_xor_sync(kFull, mt, 16));
        const float al = mt == -INFINITY ? 1.f : exp2f(m[h] - mt);
        l[h] *= al;
        m[h] = mt;
        if (kk == 0) sA[dq * H4 + h] = al;
    }
    __syncwarp();
#pragma unroll
    for (int g4 = 0; g4 < GP / 4; ++g4) {
        const float4 a = *reinterpret_cast<const float4*>(sA + g4 * 4);
        const uint64_t a01 = ptx::f2_pack(a.x, a.y), a23 = ptx::f2_pack(a.z, a.w);
#pragma unroll
        for (int e = 0; e < E; ++e) {
            acc2[g4 * 2][e] = ptx::fmul2(acc2[g4 * 2][e], a01);
            acc2[g4 * 2 + 1][e] = ptx::fmul2(acc2[g4 * 2 + 1][e], a23);
        }
    }
    if (kk == 0) {
#pragma unroll
        for (int h = 0; h < H4; ++h) {
            mw[(dq * H4 + h) * 2] = m[h];
            mw[(dq * H4 + h) * 2 + 1] = l[h];
        }
    }
#pragma unroll
    for (int gp = 0; gp < GP / 2; ++gp) {
        float lo[E], hi[E];
#pragma unroll
        for (int e = 0; e < E; ++e) ptx::f2_unpack(acc2[gp][e], lo[e], hi[e]);
        if (E == 4) {
            *reinterpret_cast<float4*>(ow + (2 * gp) * D + lane * 4) = make_float4(lo[0], lo[1], lo[2], lo[3]);
            *reinterpret_cast<float4*>(ow + (2 * gp + 1) * D + lane * 4) = make_float4(hi[0], hi[1], hi[2], hi[3]);
        } else {
            *reinterpret_cast<float2*>(ow + (2 * gp) * D + lane * 2) = make_float2(lo[0], lo[1]);
            *reinterpret_cast<float2*>(ow + (2 * gp + 1) * D + lane * 2) = make_float2(hi[0], hi[1]);
        }
    }
    __syncthreads();
    auto warp_area = [&](int w) { return sm + w * Lay::kRing; };
    if (threadIdx.x < G) {
        const int g = threadIdx.x;
        float M = -INFINITY;
        for (int w2 = 0; w2 < kW; ++w2) M = fmaxf(M, warp_area(w2)[g * 2]);
        float L = 0.f;
        for (int w2 = 0; w2 < kW; ++w2) {
            const float mw2 = warp_area(w2)[g * 2];
            const float sc = mw2 == -INFINITY ? 0.f : exp2f(mw2 - M);
            sSC[w2 * GP + g] = sc;
            L += warp_area(w2)[g * 2 + 1] * sc;
        }
        sML[g * 2] = M;
        sML[g * 2 + 1] = L;
    }
    __syncthreads();

    if (S == 1) {
        for (int i = threadIdx.x; i < G * D; i += kT) {
            const int g = i / D, d = i - g * D;
            const float M = sML[g * 2], L = sML[g * 2 + 1];
            float o = 0.f;
            if (L > 0.f) {
                for (int w2 = 0; w2 < kW; ++w2) o = fmaf(warp_area(w2)[2 * GP + g * D + d], sSC[w2 * GP + g], o);
                o /= L;
            }
            emit_f32(p, b, hk * G + g, d, o, M, L);
        }
        return;
    }

    const int slot = grp * S + split;
    for (int i = threadIdx.x; i < G * D; i += kT) {
        const int g = i / D, d = i - g * D;
        const float M = sML[g * 2], L = sML[g * 2 + 1];
        float o = 0.f;
        if (L > 0.f) {
            for (int w2 = 0; w2 < kW; ++w2) o = fmaf(warp_area(w2)[2 * GP + g * D + d], sSC[w2 * GP + g], o);
            o /= L;
        }
        p.part_o[((size_t)slot * G + g) * D + d] = o;
        if (d == 0) {
            p.part_ml[((size_t)slot * G + g) * 2] = M;
            p.part_ml[((size_t)slot * G + g) * 2 + 1] = L;
        }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = arrive_tagged(p.counters + grp, p.tag) == (unsigned)(S - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();

    // ---- last CTA of the group: merge the S slots.  Per (slot, head) scale
    // L_s * 2^(m_s - M) / L into the (now idle) stage area.
    float* ssc = sm;                      // [S][GP]
    for (int g = warp; g < G; g += kW) {
        float M = -INFINITY;
        for (int s2 = lane; s2 < S; s2 += 32) M = fmaxf(M, __ldcg(p.part_ml + ((size_t)(grp * S + s2) * G + g) * 2));
#pragma unroll
        for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(kFull, M, o));
        float L = 0.f;
        for (int s2 = lane; s2 < S; s2 += 32) {
            const float2 ml = __ldcg(reinterpret_cast<const float2*>(p.part_ml + ((size_t)(grp * S + s2) * G + g) * 2));
            const float sc = ml.x == -INFINITY ? 0.f : ml.y * exp2f(ml.x - M);
            ssc[s2 * GP + g] = sc;
            L += sc;
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) L += __shfl_xor_sync(kFull, L, o);
        if (lane == 0) {
            sML[g * 2] = M;
            sML[g * 2 + 1] = L;
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < G * D; i += kT) {
        const int g = i / D, d = i - g * D;
        const float M = sML[g * 2], L = sML[g * 2 + 1];
        float o = 0.f;
        if (L > 0.f) {
            for (int s2 = 0; s2 < S; ++s2) {
                const float sc = ssc[s2 * GP + g];
                if (sc != 0.f) o = fmaf(__ldcg(p.part_o + ((size_t)(grp * S + s2) * G + g) * D + d), sc, o);
            }
            o /= L;
        }
        emit_f32(p, b, hk * G + g, d, o, M, L);
    }
    if (threadIdx.x == 0) p.counters[grp] = 0ull;     // graph replays (same tag) start clean
}

template <int D, int GP>
int launch_f32_t(const DecodeF32Args& a, int S, const CUtensorMap& mk, const CUtensorMap& mv, int dense,
                 cudaStream_t st) {
    using Lay = F32Layout<D, GP>;
    auto kern = fog_decode_f32_kernel<D, GP>;
    // the last CTA's per-slot scales [S][GP] live in the warps' stage areas
    if (S * GP > kW * Lay::kRing) S = kW * Lay::kRing / GP;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Lay::kBytes) != cudaSuccess)
        return check_launch("paged_fog_decode (fp32): set smem attribute");
    dim3 grid(S, a.B * a.Hkv);
    kern<<<grid, kT, Lay::kBytes, st>>>(a, S, mk, mv, dense);
    return check_launch("paged_fog_decode (fp32)");
}

}  // namespace

int launch_decode_f32(const DecodeF32Args& a, cudaStream_t st) {
    const int G = a.Hq / a.Hkv;
    const int groups = a.B * a.Hkv;
    if (groups > 65535)
        return set_error(KESSIE_ERR_UNSUPPORTED, "paged_fog_decode (fp32): B * Hkv = %d above 65535", groups);
    const int max_chunks = (a.max_seq_len + 7) / 8 + 1;
    // about one CTA per SM in total, at least two chunks per warp, and no
    // more splits than the workspace has slots for
    const int sms = sm_count();
    const int s_max = max(1, min(max_chunks / (2 * kW), a.slots / groups));
    int S = min(s_max, max(1, (sms + groups - 1) / groups));
    // one CTA per SM: among the next few split counts take the one whose
    // grid fills its last wave best (equal-length groups then finish together)
    auto fill = [&](int s) {
        const long long ctas = (long long)s * groups;
        return (double)ctas / (double)(((ctas + sms - 1) / sms) * sms);
    };
    double best = fill(S);
    for (int s = S + 1; s <= min(s_max, 8 * S) && best < 0.97; ++s)
        if (fill(s) > best + 1e-9) { best = fill(s); S = s; }
    // a single wave that fills nearly as well wins: each CTA pays its ramp
    // (q, page ids, the first ring fill) and its merge once per SM instead of
    // once per wave (2 sequences at the config-3 shape: 16 groups x 9 splits
    // in one wave 344.7 us against 16 x 18 in two 355.1 us)
    const int s1 = min(s_max, sms / groups);
    if (s1 >= 1 && s1 < S && fill(s1) >= best - 0.03) S = s1;
    // K/V tiles by TMA boxes: pages (a multiple of 8 tokens) through a 5-D
    // map, a dense cache through a 4-D map that zero-fills past its end
    if (a.square_n <= 0 && a.page_size % 8)
        return set_error(KESSIE_ERR_UNSUPPORTED, "paged_fog_decode (fp32): page_size %d not a multiple of 8",
                         a.page_size);
    const int dense = a.square_n > 0 ? 1 : 0;
    const int tokens = dense ? a.square_n : a.page_size, pages = dense ? 0 : a.num_pages;
    CUtensorMap mk, mv;
    const CUresult r1 = encode_f32_kv_map(&mk, a.k_cache, a.D, tokens, a.Hkv, pages, a.token_stride, a.head_stride,
                                          a.page_stride);
    const CUresult r2 = encode_f32_kv_map(&mv, a.v_cache, a.D, tokens, a.Hkv, pages, a.token_stride, a.head_stride,
                                          a.page_stride);
    if (r1 != CUDA_SUCCESS || r2 != CUDA_SUCCESS)
        return set_error(KESSIE_ERR_ARG, "paged_fog_decode (fp32): TMA descriptor rejected (%d/%d)", (int)r1, (int)r2);
    if (a.D == 128) {
        if (G <= 4) return launch_f32_t<128, 4>(a, S, mk, mv, dense, st);
        if (G <= 8) return launch_f32_t<128, 8>(a, S, mk, mv, dense, st);
        return launch_f32_t<128, 16>(a, S, mk, mv, dense, st);
    }
    if (G <= 4) return launch_f32_t<64, 4>(a, S, mk, mv, dense, st);
    if (G <= 8) return launch_f32_t<64, 8>(a, S, mk, mv, dense, st);
    return launch_f32_t<64, 16>(a, S, mk, mv, dense, st);
}

}  // namespace kessie
