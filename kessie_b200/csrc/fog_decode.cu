// fog_decode.cu -- paged fog-attention decode: persistent split-KV kernel with
// the split merge (and, for context parallelism, the cross-GPU push) fused in.
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
//   work  = the visible 16-token units of every (seq, kv_head) group, laid
//           end to end (group g = b*Hkv + hk).  The grid is one wave of
//           persistent CTAs (occupancy x SMs); CTA i takes the contiguous
//           range [i*W, (i+1)*W) with W = ceil(total / grid), so every CTA
//           streams the same number of KV bytes whatever the sequence
//           lengths -- no tail wave.  The ranges are derived on the device
//           from seq_lens, so the launch needs no host synchronisation.
//           A CTA's range splits into "segments", one per group it touches;
//           each KV byte is read once for all Hq/Hkv query heads (GQA).
//   CTA   = 1 producer warp + 4 consumer warps + 1 helper warp.  The producer prefetches page
//           ids 128 units ahead (registers -> smem window) and issues one TMA
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
//   merge = at a segment end the 4 warps merge pairwise through smem and the
//           CTA writes one partial (O/l, m, l) per query head into slot
//           (cta + group) of the workspace -- unique, because ranges are
//           ordered -- and bumps the group's arrival counter (tagged with a
//           per-launch number, so leftover workspace contents never count).  The CTA that
//           arrives last merges the group's partials (about grid/groups + 1
//           of them) and writes out / out_partial, or (context parallelism)
//           stores the rows into every rank's exchange buffer over NVLink as
//           self-validating (value, epoch) words -- no fence, no flag, so the
//           storing CTA never waits on the remote stores (cp_layout.cuh).
//           The merging CTA also zeroes the counter, so graph replays (same
//           tag) start clean.  A segment that ends inside the CTA's range
//           (its group continues in the next CTA) is handed to the helper
//           warp through a shared-memory staging area: the helper stores the
//           partial, fences, arrives and merges if it was last, while the
//           consumers go on streaming.  Under a saturated memory system that
//           fence took ~5 us, and the CTAs that switch groups were the last to
//           finish.
//   cp    = cp_combine_kernel polls its own exchange buffer (bounded) until
//           every rank's words of a row carry the step's epoch, then merges
//           the world shard results.  One decode kernel and one small combine
//           per step, no collective library call.
//   launch = programmatic dependent launches (cudaLaunchKernelEx).  When the
//           launch registry shows that the preceding programmatic launch on
//           the stream wrote none of q, the cache, the tables, the lengths or
//           the bias bitmap, everything up to a CTA's first global store runs
//           before griddepcontrol.wait, so a step's ramp overlaps the previous
//           step's tail; the combine lets the next step start at its own start.
#include "common.cuh"
#include "cp_layout.cuh"
#include "decode_f32.cuh"
#include "fog_bias.cuh"
#include "ptx.cuh"
#include "tma_host.cuh"

#include <math.h>

#include <atomic>
#include <mutex>
#include <type_traits>

namespace kessie {
namespace {

constexpr int kNCW = 4;          // consumer warps
constexpr uint64_t kSpinNs = 2000000000ull;   // bound of an mbarrier wait with nothing ahead of it
constexpr uint64_t kSpinMaxNs = 32000000000ull; // cap when a preceding combine's delay is added
constexpr int kNST = 3;          // pipeline stages
constexpr int kIdWin = 128;      // page ids per prefetch window (units)
constexpr int kHelperWarp = kNCW + 1;  // finishes mid-range segment ends for the consumers
constexpr int kThreads = (kNCW + 2) * 32;
constexpr int kCtasPerSm = 2;    // upper bound used to size the workspace
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
    int units_per_page, num_pages, max_units;
    float* part_o;        // [slots][G][D]   segment partial O/l
    float* part_ml;       // [slots][G][2]   (m in log2 units, l)
    unsigned long long* counters;   // [B*Hkv] (launch tag << 32) | arrivals, per group
    uint32_t tag;         // this launch's tag (non-zero); a counter with another tag counts as zero
    void* out;            // [B][Hq][D] q dtype, or null
    float* out_part;      // [B][Hq][D+2] (O/l, ln m, l), or null
    CpLink cp;            // cp.world > 0: push merged rows into every rank's exchange buffer
    FogBias bias;         // additive fog bias on the scores (vLLM path), bias.on == 0: none
    int* status;
    int early;            // read ahead of griddepcontrol.wait (every global store still follows it)
    uint64_t spin_ns;     // bound of each mbarrier wait (longer when early: see run_decode)
    const void* ws_base;  // host side: the workspace's byte range, for the launch registry
    size_t ws_bytes;
};

// Visible local key range of one sequence.
struct SeqInfo {
    int k_lo, k_hi, off;  // keys [k_lo, k_hi) of the local shard; global position of key 0
    int qp;               // query position (global); the sequence holds qp + 1 keys in total
    int ulo, n;           // first visible 16-token unit and the unit count (0: nothing visible)
};

__device__ __forceinline__ SeqInfo seq_info(const DecodeParams& p, int b) {
    SeqInfo s;
    int n = p.seq_lens[b];
    if (n < 0 || n > p.max_units * 16) {
        record_status(p.status, KESSIE_DEV_BAD_ARG);
        n = n < 0 ? 0 : p.max_units * 16;
    }
    s.off = p.kv_off ? p.kv_off[b] : 0;
    const int qp = p.q_pos ? p.q_pos[b] : s.off + n - 1;
    s.qp = qp;
    s.k_hi = min(n, qp - s.off + 1);
    s.k_lo = p.window > 0 ? max(0, qp - p.window + 1 - s.off) : 0;
    if (s.k_hi > s.k_lo) {
        s.ulo = s.k_lo >> 4;
        s.n = ((s.k_hi + 15) >> 4) - s.ulo;
    } else {
        s.ulo = 0;
        s.n = 0;
    }
    return s;
}

// Fog weight of the key at global position j (kessie_hip_kernels.py:408-412).
// (j / (cs-1))^alpha as 2^(alpha * log2(j * inv_den)) on the special-function
// unit (relative error ~1e-6, far below the bf16 rounding of P): a handful of
// instructions instead of an IEEE divide and an accurate powf per key, which
// keeps the decode HBM-bound when the SM clock drops under the power cap.
__device__ __forceinline__ float fog_weight(const DecodeParams& p, int cs, float inv_den, int j) {
    if (p.fog_w) return __ldg(p.fog_w + j);
    if (j >= cs) return 1.f;
    return ptx::ex2(p.fog_alpha * ptx::lg2((float)j * inv_den));
}

template <int D, int NT>
struct Smem {
    static constexpr int kTile = 16 * D * 2;              // bytes of one 16-token K (or V) slice
    static constexpr int kStage = kNCW * 2 * kTile;
    static constexpr int QP = NT * 8;                     // padded query columns
    static constexpr int kMrgFloats = D * QP + 2 * QP;    // one warp's (acc, m, l)
    static constexpr int kMrgOff = kNST * kStage;
    static constexpr int kIdsOff = kMrgOff + 2 * kMrgFloats * 4;
    static constexpr int kMetaOff = kIdsOff + kIdWin * 4;
    static constexpr int kBarOff = (kMetaOff + kNST * kNCW * 4 + 7) & ~7;   // full[kNST], empty[kNST], job_full, job_empty
    static constexpr int kCtlOff = kBarOff + (2 * kNST + 2) * 8;
    static constexpr int kStgOff = (kCtlOff + 16 * 4 + 15) & ~15;           // handed-off partial: [QP][D] O/l, [QP][2] (m, l)
    static constexpr int kBytes = kStgOff + QP * (D + 2) * 4;
    static constexpr int kAlloc = kBytes + 1024;          // 1 KB slack for 1024-byte alignment
};

// Byte offset of (row r, 16B chunk c) inside a 128B-swizzled tile.
__device__ __forceinline__ uint32_t swz(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ int par_of(uint32_t epoch) { return (int)(epoch & 1u); }

__device__ __forceinline__ void consumers_sync() {
    asm volatile("bar.sync 1, %0;" :: "r"(kNCW * 32) : "memory");
}

// Walks the segments of one CTA's unit range in order.  Every warp runs its
// own copy (the loads are warp-uniform broadcasts).
struct Segment {
    int g;        // group = b * Hkv + hk
    int u0, nu;   // first unit (sequence-local) and unit count of the segment
    int gstart;   // flattened position of the group's first unit
    int gn;       // units of the whole group
    SeqInfo si;
};

struct SegWalker {
    int g, off, pos, end, cur_b;
    SeqInfo si;

    __device__ void init(const DecodeParams& p, int g0, int off0, int u_begin, int u_end) {
        g = g0; off = off0; pos = u_begin; end = u_end; cur_b = -1;
        if (g0 >= 0) { cur_b = g0 / p.Hkv; si = seq_info(p, cur_b); }
        else pos = end;
    }
    __device__ bool next(const DecodeParams& p, Segment& s) {
        while (pos < end) {
            if (off < si.n) {
                const int cnt = min(si.n - off, end - pos);
                s.g = g; s.u0 = si.ulo + off; s.nu = cnt; s.gstart = pos - off; s.gn = si.n; s.si = si;
                pos += cnt; off += cnt;
                return true;
            }
            if (++g >= p.B * p.Hkv) { pos = end; break; }
            off = 0;
            const int b = g / p.Hkv;
            if (b != cur_b) { cur_b = b; si = seq_info(p, b); }
        }
        return false;
    }
};

template <bool BF16>
__device__ __forceinline__ void store_out_row(void* out, int64_t idx, const float* o, int E) {
    using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
    T* dst = static_cast<T*>(out) + idx;
    if (E == 4) {
        uint2 v;
        v.x = ptx::pack2<BF16>(o[0], o[1]);
        v.y = ptx::pack2<BF16>(o[2], o[3]);
        *reinterpret_cast<uint2*>(dst) = v;
    } else {
        *reinterpret_cast<uint32_t*>(dst) = ptx::pack2<BF16>(o[0], o[1]);
    }
}

// One merged row: lane holds o[d] for d = lane*E .. lane*E+E-1 (normalised),
// M (log2 units, -inf when nothing was visible) and L.
template <int D, bool BF16>
__device__ __forceinline__ void emit_row(const DecodeParams& p, int row, int lane, const float (&o)[D / 32],
                                         float M, float L) {
    constexpr int E = D / 32;
    const int d0 = lane * E;
    if (p.out) store_out_row<BF16>(p.out, (int64_t)row * D + d0, o, E);
    if (p.out_part) {
        float* dst = p.out_part + (int64_t)row * (D + 2);
#pragma unroll
        for (int e = 0; e < E; e += 2) *reinterpret_cast<float2*>(dst + d0 + e) = make_float2(o[e], o[e + 1]);
        if (lane == 0) *reinterpret_cast<float2*>(dst + D) = make_float2(M == -INFINITY ? -INFINITY : M * kLn2, L);
    }
    if (p.cp.world > 0) {
        const CpLayout lay{p.cp.world, p.B * p.Hq, D};
        const int par = par_of(p.cp.epoch);
        const uint32_t ep = p.cp.epoch;
#pragma unroll
        for (int r = 0; r < kCpMaxRanks; ++r) {
            if (r >= p.cp.world) break;
            uint64_t* w = lay.row(p.cp.peer[r], par, p.cp.rank, row);
#pragma unroll
            for (int e = 0; e < E; e += 2)
                *reinterpret_cast<ulonglong2*>(w + d0 + e) = make_ulonglong2(cp_word(o[e], ep), cp_word(o[e + 1], ep));
            if (lane == 0) *reinterpret_cast<ulonglong2*>(w + D) = make_ulonglong2(cp_word(M, ep), cp_word(L, ep));
        }
    }
}

// Merge the K segment partials of group g (slots first+g .. first+K-1+g) and
// emit its G rows; K == 0 emits empty rows.  Run by `nw` warps (warp index
// `warp` among them): the 4 consumer warps, or the helper warp alone.
template <int D, bool BF16>
__device__ void merge_and_emit(const DecodeParams& p, int g, int first, int K, int warp, int lane, int nw = kNCW) {
    constexpr int E = D / 32;
    const int b = g / p.Hkv, hk = g - b * p.Hkv;
    const size_t sstride = (size_t)p.G * D;
    for (int q = warp; q < p.G; q += nw) {
        float M = -INFINITY;
        for (int k = lane; k < K; k += 32) M = fmaxf(M, __ldcg(p.part_ml + ((size_t)(first + k + g) * p.G + q) * 2));
        M = warp_max(M);
        float L = 0.f, acc[E];
#pragma unroll
        for (int e = 0; e < E; ++e) acc[e] = 0.f;
        if (M != -INFINITY) {
            for (int kb = 0; kb < K; kb += 32) {
                const int k = kb + lane;
                float w = 0.f;
                if (k < K) {
                    const float2 ml = __ldcg(reinterpret_cast<const float2*>(p.part_ml + ((size_t)(first + k + g) * p.G + q) * 2));
                    w = ml.y * exp2f(ml.x - M);
                }
                L += w;
                const int n = min(32, K - kb);
                const float* base = p.part_o + ((size_t)(first + kb + g) * p.G + q) * D + lane * E;
#pragma unroll 8
                for (int j = 0; j < n; ++j) {
                    const float wj = __shfl_sync(0xffffffffu, w, j);
                    const float* pc = base + (size_t)j * sstride;
                    if (E == 4) {
                        const float4 x = __ldcg(reinterpret_cast<const float4*>(pc));
                        acc[0] += wj * x.x; acc[1] += wj * x.y; acc[2] += wj * x.z; acc[3] += wj * x.w;
                    } else {
                        const float2 x = __ldcg(reinterpret_cast<const float2*>(pc));
                        acc[0] += wj * x.x; acc[1] += wj * x.y;
                    }
                }
            }
            L = warp_sum(L);
        }
        float o[E];
#pragma unroll
        for (int e = 0; e < E; ++e) o[e] = L > 0.f ? acc[e] / L : 0.f;
        emit_row<D, BF16>(p, b * p.Hq + hk * p.G + q, lane, o, M, L);
    }
}

// Count one arrival at a group counter; returns the arrivals before this one
// (a counter holding another launch's tag, or garbage, counts as zero).
__device__ __forceinline__ unsigned arrive(unsigned long long* c, uint32_t tag) {
    const unsigned long long hi = (unsigned long long)tag << 32;
    unsigned long long old = *reinterpret_cast<volatile unsigned long long*>(c);
    while (true) {
        const unsigned long long cur = (old >> 32) == tag ? old : hi;
        const unsigned long long prev = atomicCAS(c, old, cur + 1ull);
        if (prev == old) return (unsigned)(cur & 0xffffffffull);
        old = prev;
    }
}

template <int D, bool BF16, int NT>
__global__ void __launch_bounds__(kThreads, NT == 1 ? 2 : 1) fog_decode_kernel(const __grid_constant__ CUtensorMap tmK,
                                                                  const __grid_constant__ CUtensorMap tmV,
                                                                  const DecodeParams p) {
    using S = Smem<D, NT>;
    constexpr int QP = S::QP;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    int32_t* idw = reinterpret_cast<int32_t*>(smem + S::kIdsOff);
    int32_t* meta = reinterpret_cast<int32_t*>(smem + S::kMetaOff);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kBarOff);
    uint64_t* empty = full + kNST;
    uint64_t* job_full = empty + kNST;     // a mid-range segment's partial is staged for the helper
    uint64_t* job_empty = job_full + 1;    // the helper is done with the staging
    float* stg = reinterpret_cast<float*>(smem + S::kStgOff);
    int* ctl = reinterpret_cast<int*>(smem + S::kCtlOff);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Programmatic dependent launch.  Without p.early every thread waits here
    // for the preceding grid.  With it (the host found that the preceding
    // programmatic launches wrote none of q, the cache, the tables or the
    // lengths) the range search, page ids, TMA loads and the math run ahead,
    // and each thread waits before its first global store: the consumers at
    // their final segment (mid-range ends only stage into shared memory) or
    // before emitting an empty group, the helper before its first partial.
    // While one warp sits in that wait another may wait on it through an
    // mbarrier, so those waits are bounded by p.spin_ns, which covers how long
    // the preceding grid can still run.
    if (!p.early) ptx::grid_dependency_wait();

    // ---------------------------------------------------------------- range of this CTA
    if (threadIdx.x == 0) {
        for (int s = 0; s < kNST; ++s) { ptx::mbar_init(&full[s], 1); ptx::mbar_init(&empty[s], kNCW); }
        ptx::mbar_init(job_full, 1);
        ptx::mbar_init(job_empty, 1);
        ptx::fence_mbar_init();
    }
    if (warp == kNCW) {
        int tot = 0;
        for (int base = 0; base < p.B; base += 32) {
            const int b = base + lane;
            if (b < p.B) tot += seq_info(p, b).n;
        }
        tot = __reduce_add_sync(0xffffffffu, tot) * p.Hkv;
        const int W = tot > 0 ? (tot + (int)gridDim.x - 1) / (int)gridDim.x : 0;
        const int U0 = (int)blockIdx.x * W;
        int g0 = -1, off0 = 0;
        if (U0 < tot) {
            int acc = 0;
            for (int base = 0; base < p.B; base += 32) {
                const int b = base + lane;
                const int n = b < p.B ? seq_info(p, b).n : 0;
                const int v = n * p.Hkv;
                int incl = v;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int x = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += x;
                }
                const bool hit = v > 0 && acc + incl - v <= U0 && U0 < acc + incl;
                const unsigned bal = __ballot_sync(0xffffffffu, hit);
                if (bal) {
                    const int src = __ffs(bal) - 1;
                    const int pre = acc + __shfl_sync(0xffffffffu, incl - v, src);
                    const int nb = __shfl_sync(0xffffffffu, n, src);
                    const int rel = U0 - pre;
                    const int hk = rel / nb;
                    g0 = (base + src) * p.Hkv + hk;
                    off0 = rel - hk * nb;
                    break;
                }
                acc += __shfl_sync(0xffffffffu, incl, 31);
            }
        }
        if (lane == 0) {
            ctl[0] = W; ctl[1] = tot; ctl[2] = g0; ctl[3] = off0;
        }
    }
    __syncthreads();
    const int W = ctl[0], tot = ctl[1];
    const int U0 = (int)blockIdx.x * W;
    const int U1 = min(tot, U0 + W);
    SegWalker walk;
    walk.init(p, ctl[2], ctl[3], U0, U1);

    // ---------------------------------------------------------------- producer
    if (warp == kNCW) {
        const uint64_t pol = ptx::policy_evict_first();
        if (lane == 0) { ptx::prefetch_tensormap(&tmK); ptx::prefetch_tensormap(&tmV); }
        int itg = 0;
        bool broken = false;
        Segment sg;
        while (!broken && walk.next(p, sg)) {
            const int b = sg.g / p.Hkv, hk = sg.g - b * p.Hkv;
            const int32_t* bt = p.block_table + (int64_t)b * p.bt_stride;
            int nx[kIdWin / 32];
            auto fetch = [&](int wbase) {
#pragma unroll
                for (int k = 0; k < kIdWin / 32; ++k) {
                    const int i = wbase + lane + 32 * k;
                    nx[k] = i < sg.nu ? __ldg(bt + (sg.u0 + i) / p.units_per_page) : INT_MIN;
                }
            };
            auto publish = [&]() {
#pragma unroll
                for (int k = 0; k < kIdWin / 32; ++k) {
                    int id = nx[k];
                    if (id != INT_MIN && (id < 0 || id >= p.num_pages)) {
                        record_status(p.status, KESSIE_DEV_BAD_PAGE_ID);
                        id = -1;
                    }
                    idw[lane + 32 * k] = id;
                }
            };
            fetch(0);
            __syncwarp();
            publish();
            __syncwarp();
            fetch(kIdWin);
            int wbase = 0;
            const int n_iter = (sg.nu + kNCW - 1) / kNCW;
            for (int it = 0; it < n_iter; ++it, ++itg) {
                if (it * kNCW - wbase >= kIdWin) {
                    __syncwarp();
                    publish();
                    __syncwarp();
                    wbase += kIdWin;
                    fetch(wbase + kIdWin);
                }
                const int s = itg % kNST;
                bool ok = true;
                if (lane == 0 && itg >= kNST) ok = ptx::mbar_wait(&empty[s], ((uint32_t)(itg / kNST) & 1u) ^ 1u, p.spin_ns);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) {
                    if (lane == 0) record_status(p.status, KESSIE_DEV_WAIT_TIMEOUT);
                    broken = true;
                    break;
                }
                if (lane == 0) {
                    const int nu_it = min(kNCW, sg.nu - it * kNCW);
                    uint8_t* st = smem + s * S::kStage;
                    for (int w = 0; w < nu_it; ++w) meta[s * kNCW + w] = idw[it * kNCW + w - wbase];
                    ptx::mbar_arrive_expect_tx(&full[s], (uint32_t)(nu_it * 2 * S::kTile));
                    for (int w = 0; w < nu_it; ++w) {
                        const int u = sg.u0 + it * kNCW + w;
                        const int id = meta[s * kNCW + w];
                        const int page = id < 0 ? p.num_pages : id;          // out of range -> zero fill
                        const int tok0 = (u % p.units_per_page) * 16;
                        ptx::tma_load_5d_hint(st + w * 2 * S::kTile, &tmK, &full[s], 0, tok0, 0, hk, page, pol);
                        ptx::tma_load_5d_hint(st + w * 2 * S::kTile + S::kTile, &tmV, &full[s], 0, tok0, 0, hk, page, pol);
                    }
                }
            }
        }
        // drain: every issued load has landed before this warp exits
        if (lane == 0) {
            for (int it = max(0, itg - kNST); it < itg; ++it) {
                if (!ptx::mbar_wait(&full[it % kNST], (uint32_t)(it / kNST) & 1u, p.spin_ns)) {
                    record_status(p.status, KESSIE_DEV_WAIT_TIMEOUT);
                    break;
                }
            }
        }
        return;
    }

    // ---------------------------------------------------------------- helper
    // A segment that ends inside the CTA's range (its group continues in the
    // next CTA) is finished here, off the consumers' path: the consumers
    // stage the normalised partial in shared memory and go on with the next
    // segment, while this warp stores the partial, fences, counts the
    // arrival and, if it was the group's last, merges the group alone.
    // Under a saturated memory system the fence alone took several us.
    if (warp == kHelperWarp) {
        bool waited = !p.early;
        for (int job = 0;; ++job) {
            // lane 0 waits (the warp may idle for most of the launch); the
            // warp barrier orders the other lanes' reads after it
            bool ok = true;
            if (lane == 0) ok = ptx::mbar_wait(job_full, (uint32_t)job & 1u, p.spin_ns);
            __syncwarp();
            if (!__shfl_sync(0xffffffffu, ok, 0)) {
                if (lane == 0) record_status(p.status, KESSIE_DEV_WAIT_TIMEOUT);
                break;
            }
            const int slot = ctl[8], g = ctl[9], first = ctl[10], K = ctl[11];
            if (slot < 0) break;                                    // no more segments
            if (!waited) {
                ptx::grid_dependency_wait();
                waited = true;
            }
            const int G = p.G;
            float4* po = reinterpret_cast<float4*>(p.part_o + (size_t)slot * G * D);
            const float4* so = reinterpret_cast<const float4*>(stg);
            for (int i = lane; i < G * D / 4; i += 32) po[i] = so[i];
            for (int i = lane; i < 2 * G; i += 32) p.part_ml[(size_t)slot * G * 2 + i] = stg[S::QP * D + i];
            __threadfence();
            __syncwarp();
            int last = 0;
            if (lane == 0) last = arrive(p.counters + g, p.tag) == (unsigned)(K - 1);
            last = __shfl_sync(0xffffffffu, last, 0);
            if (last) {
                __threadfence();
                if (lane == 0) p.counters[g] = 0ull;
                merge_and_emit<D, BF16>(p, g, first, K, 0, lane, 1);
            }
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(job_empty);
        }
        return;
    }

    // ---------------------------------------------------------------- consumers
    // Groups with no visible key anywhere in this shard still produce rows
    // (zeros; m = -inf, l = 0); CTA g % grid emits them.
    bool waited = !p.early;
    for (int g = blockIdx.x; g < p.B * p.Hkv; g += gridDim.x) {
        if (seq_info(p, g / p.Hkv).n == 0) {
            if (!waited) {
                ptx::grid_dependency_wait();
                waited = true;
            }
            merge_and_emit<D, BF16>(p, g, 0, 0, warp, lane);
        }
    }

    const int g8 = lane >> 2, t = lane & 3;
    const int mi = lane >> 3, rr = lane & 7;
    const int k_key = rr + 8 * (mi & 1), k_cadd = mi >> 1;     // ldmatrix rows for K (non-trans)
    const int v_key = rr + 8 * (mi >> 1), v_cadd = mi & 1;     // ldmatrix rows for V (trans)
    float* mrg = reinterpret_cast<float*>(smem + S::kMrgOff);  // [2][D*QP + 2*QP]
    int itg = 0;
    int njobs = 0;                         // segments handed to the helper
    bool broken = false;
    Segment sg;
    while (walk.next(p, sg)) {
        const int b = sg.g / p.Hkv, hk = sg.g - b * p.Hkv;
        const int k_lo = sg.si.k_lo, k_hi = sg.si.k_hi, off = sg.si.off;
        // Q^T B-fragments: b0 = Q[q=g8][kk*16+2t..+1], b1 = Q[g8][kk*16+2t+8..+9]
        uint32_t qf[NT][D / 16][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int qh = nt * 8 + g8;
            const bool ok = qh < p.G;
            const uint16_t* qrow = reinterpret_cast<const uint16_t*>(p.q) + (int64_t)b * p.q_sb +
                                   (int64_t)(hk * p.G + (ok ? qh : 0)) * p.q_sh;
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
                qf[nt][kk][0] = ok ? *reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 2 * t) : 0u;
                qf[nt][kk][1] = ok ? *reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 2 * t + 8) : 0u;
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
        const float inv_den = 1.f / (float)max(cs - 1, 1);
        const bool has_bias = p.bias.on != 0;
        const int bias_fb = has_bias ? fog_bias_boundary(p.bias, sg.si.qp + 1) : 0;

        const int n_iter = (sg.nu + kNCW - 1) / kNCW;
        for (int it = 0; it < n_iter; ++it, ++itg) {
            const int s = itg % kNST;
            if (!broken) {
                const bool ok = ptx::mbar_wait(&full[s], (uint32_t)(itg / kNST) & 1u, p.spin_ns);
                if (!__all_sync(0xffffffffu, ok)) {
                    if (lane == 0) record_status(p.status, KESSIE_DEV_WAIT_TIMEOUT);
                    broken = true;
                }
            }
            const int i = it * kNCW + warp;
            if (!broken && i < sg.nu) {
                uint8_t* ktile = smem + s * S::kStage + warp * 2 * S::kTile;
                uint8_t* vtile = ktile + S::kTile;
                const int u = sg.u0 + i;
                const int j0 = u * 16;                         // local index of key 0 of the unit
                const bool page_ok = meta[s * kNCW + warp] >= 0;
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
                const int ja = j0 + g8, jb = j0 + g8 + 8;
                const bool va = page_ok && ja >= k_lo && ja < k_hi;
                const bool vb = page_ok && jb >= k_lo && jb < k_hi;
                float wa = 1.f, wb = 1.f;
                if (has_fog) {      // only visible keys: fog_weights covers visible positions only
                    wa = va ? fog_weight(p, cs, inv_den, off + ja) : 0.f;
                    wb = vb ? fog_weight(p, cs, inv_den, off + jb) : 0.f;
                }
                float ba = 0.f, bb2 = 0.f;   // additive bias, log2 units
                if (has_bias) {
                    ba = va ? fog_bias_at(p.bias, bias_fb, off + ja) * kLog2e : 0.f;
                    bb2 = vb ? fog_bias_at(p.bias, bias_fb, off + jb) * kLog2e : 0.f;
                }
                uint32_t pb0[NT], pb1[NT];
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    const float s00 = va ? fmaf(sacc[nt][0], p.scale_log2, ba) : -INFINITY;
                    const float s01 = va ? fmaf(sacc[nt][1], p.scale_log2, ba) : -INFINITY;
                    const float s10 = vb ? fmaf(sacc[nt][2], p.scale_log2, bb2) : -INFINITY;
                    const float s11 = vb ? fmaf(sacc[nt][3], p.scale_log2, bb2) : -INFINITY;
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
            if (lane == 0 && !broken) ptx::mbar_arrive(&empty[s]);
        }

        // ------------------------------------------------------------ segment end
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int j = 0; j < 2; ++j)
#pragma unroll
                for (int o = 4; o < 32; o <<= 1) l[nt][j] += __shfl_xor_sync(0xffffffffu, l[nt][j], o);

        // pairwise merge of the 4 warps' states: 2,3 -> 0,1, then 1 -> 0
        auto put = [&](float* r) {
            float* rm = r + D * QP;
            float* rl = rm + QP;
            if (g8 == 0) {
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    rm[nt * 8 + 2 * t] = m[nt][0]; rm[nt * 8 + 2 * t + 1] = m[nt][1];
                    rl[nt * 8 + 2 * t] = l[nt][0]; rl[nt * 8 + 2 * t + 1] = l[nt][1];
                }
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int mt = 0; mt < D / 16; ++mt) {
                    float* o = r + (mt * 16 + g8) * QP + nt * 8 + 2 * t;
                    o[0] = acc[nt][mt][0]; o[1] = acc[nt][mt][1];
                    o[8 * QP] = acc[nt][mt][2]; o[8 * QP + 1] = acc[nt][mt][3];
                }
        };
        auto take = [&](const float* r) {
            const float* rm = r + D * QP;
            const float* rl = rm + QP;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                float sa[2], sb[2];
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const int q = nt * 8 + 2 * t + j;
                    const float mo = rm[q], lo = rl[q];
                    const float mn = fmaxf(m[nt][j], mo);
                    const float base = mn == -INFINITY ? 0.f : mn;
                    sa[j] = exp2f(m[nt][j] - base);
                    sb[j] = exp2f(mo - base);
                    l[nt][j] = l[nt][j] * sa[j] + lo * sb[j];
                    m[nt][j] = mn;
                }
#pragma unroll
                for (int mt = 0; mt < D / 16; ++mt) {
                    const float* o = r + (mt * 16 + g8) * QP + nt * 8 + 2 * t;
                    acc[nt][mt][0] = acc[nt][mt][0] * sa[0] + o[0] * sb[0];
                    acc[nt][mt][1] = acc[nt][mt][1] * sa[1] + o[1] * sb[1];
                    acc[nt][mt][2] = acc[nt][mt][2] * sa[0] + o[8 * QP] * sb[0];
                    acc[nt][mt][3] = acc[nt][mt][3] * sa[1] + o[8 * QP + 1] * sb[1];
                }
            }
        };
        if (!waited && walk.pos >= walk.end) {              // the final segment's stores follow the wait
            ptx::grid_dependency_wait();
            waited = true;
        }
        consumers_sync();                                   // region free from the previous segment
        if (warp >= 2) put(mrg + (warp - 2) * S::kMrgFloats);
        consumers_sync();
        if (warp < 2) take(mrg + warp * S::kMrgFloats);
        consumers_sync();
        if (warp == 1) put(mrg);
        consumers_sync();
        const int slot = (int)blockIdx.x + sg.g;
        const int first = sg.gstart / W;
        const int K = (sg.gstart + sg.gn - 1) / W - first + 1;
        const bool final_seg = walk.pos >= walk.end;
        if (warp == 0) {
            take(mrg);
            // a mid-range segment goes to the helper: wait until it has
            // released the staging (bounded), stage, hand over
            if (!final_seg && njobs > 0 &&
                !__all_sync(0xffffffffu, ptx::mbar_wait(job_empty, (uint32_t)(njobs - 1) & 1u, p.spin_ns))) {
                if (lane == 0) record_status(p.status, KESSIE_DEV_WAIT_TIMEOUT);
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const int q = nt * 8 + 2 * t + j;
                    if (q < p.G) {
                        float* po = final_seg ? p.part_o + ((size_t)slot * p.G + q) * D : stg + q * D;
                        float* pm = final_seg ? p.part_ml + ((size_t)slot * p.G + q) * 2 : stg + S::QP * D + q * 2;
                        const float L = l[nt][j];
#pragma unroll
                        for (int mt = 0; mt < D / 16; ++mt) {
                            po[mt * 16 + g8] = L > 0.f ? acc[nt][mt][j] / L : 0.f;
                            po[mt * 16 + g8 + 8] = L > 0.f ? acc[nt][mt][2 + j] / L : 0.f;
                        }
                        if (g8 == 0) *reinterpret_cast<float2*>(pm) = make_float2(m[nt][j], L);
                    }
                }
            if (final_seg) {
                __threadfence();
            } else {
                __syncwarp();
                if (lane == 0) {
                    ctl[8] = slot; ctl[9] = sg.g; ctl[10] = first; ctl[11] = K;
                    ptx::mbar_arrive(job_full);
                }
            }
        }
        if (!final_seg) {
            ++njobs;
            continue;
        }
        consumers_sync();
        ptx::launch_dependents();                            // last segment: the cp combine may start
        if (threadIdx.x == 0) ctl[5] = arrive(p.counters + sg.g, p.tag) == (unsigned)(K - 1);
        consumers_sync();
        if (ctl[5]) {
            __threadfence();
            if (threadIdx.x == 0) p.counters[sg.g] = 0ull;
            merge_and_emit<D, BF16>(p, sg.g, first, K, warp, lane);
        }
    }
    // the helper stops once it has finished the last segment handed to it
    if (warp == 0) {
        if (njobs > 0 && !__all_sync(0xffffffffu, ptx::mbar_wait(job_empty, (uint32_t)(njobs - 1) & 1u, p.spin_ns))) {
            if (lane == 0) record_status(p.status, KESSIE_DEV_WAIT_TIMEOUT);
        }
        if (lane == 0) {
            ctl[8] = -1;
            ptx::mbar_arrive(job_full);
        }
    }
    // a CTA with nothing to store still ends after the preceding grid, so
    // that this grid's completion (or signal) implies that grid's completion
    if (!waited) ptx::grid_dependency_wait();
}

// Context-parallel combine: one warp per output row (4 rows per CTA), reading
// only this rank's exchange buffer.  Every lane polls (bounded by wait_ns) its
// slice of the row from all world sources until each word carries the epoch;
// the m, l words ride with lane 0's slice.  Then a warp reduction and the LSE
// merge.
struct CpCombineParams {
    void* buf;            // this rank's exchange buffer
    CpLayout lay;
    int Hq;
    uint32_t epoch;
    int64_t wait_ns;
    void* out;
    float* out_part;
    int* status;
};

template <int D, bool BF16>
__global__ void __launch_bounds__(128) cp_combine_kernel(const CpCombineParams a) {
    constexpr int E = D / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * 4 + warp;
    // The next step's decode may start now, while this step's decode CTAs
    // finish: its stores follow its own wait for this grid, whose block 0
    // waits for the decode at the end.
    ptx::launch_dependents();
    if (row >= a.lay.rows) return;
    const int par = par_of(a.epoch);
    const int world = a.lay.world;
    const uint32_t ep = a.epoch;
    float x[kCpMaxRanks][E], ms[kCpMaxRanks], ls[kCpMaxRanks];
    bool ok = true;
    uint64_t t0 = 0;
#pragma unroll
    for (int s = 0; s < kCpMaxRanks; ++s) {
        if (s >= world || !ok) break;
        const uint64_t* w = a.lay.row(a.buf, par, s, row);
        while (true) {
            uint64_t v[E], m2[2];
#pragma unroll
            for (int e = 0; e < E; e += 2) ptx::ld_volatile_v2u64(w + lane * E + e, v[e], v[e + 1]);
            ptx::ld_volatile_v2u64(w + D, m2[0], m2[1]);
            bool ready = (uint32_t)(m2[0] >> 32) == ep && (uint32_t)(m2[1] >> 32) == ep;
#pragma unroll
            for (int e = 0; e < E; ++e) ready = ready && (uint32_t)(v[e] >> 32) == ep;
            if (__all_sync(0xffffffffu, ready)) {
#pragma unroll
                for (int e = 0; e < E; ++e) x[s][e] = __uint_as_float((uint32_t)v[e]);
                ms[s] = __uint_as_float((uint32_t)m2[0]);
                ls[s] = __uint_as_float((uint32_t)m2[1]);
                break;
            }
            // the give-up decision is warp-uniform: every lane leaves together
            bool late = false;
            if (t0 == 0) t0 = ptx::globaltimer_ns();
            else late = ptx::globaltimer_ns() - t0 > (uint64_t)a.wait_ns;
            if (__any_sync(0xffffffffu, late)) { ok = false; break; }
        }
    }
    if (!ok && lane == 0) record_status(a.status, KESSIE_DEV_WAIT_TIMEOUT);
    float M = -INFINITY, L = 0.f, acc[E];
#pragma unroll
    for (int e = 0; e < E; ++e) acc[e] = 0.f;
    if (ok) {
#pragma unroll
        for (int s = 0; s < kCpMaxRanks; ++s)
            if (s < world) M = fmaxf(M, ms[s]);
        if (M != -INFINITY) {
#pragma unroll
            for (int s = 0; s < kCpMaxRanks; ++s) {
                if (s < world) {
                    const float ws = ls[s] * exp2f(ms[s] - M);
                    L += ws;
#pragma unroll
                    for (int e = 0; e < E; ++e) acc[e] += ws * x[s][e];
                }
            }
        }
    }
    float o[E];
#pragma unroll
    for (int e = 0; e < E; ++e) o[e] = L > 0.f ? acc[e] / L : 0.f;
    if (!ok) { M = -INFINITY; L = 0.f; }
    if (a.out) store_out_row<BF16>(a.out, (int64_t)row * D + lane * E, o, E);
    if (a.out_part) {
        float* dst = a.out_part + (int64_t)row * (D + 2);
#pragma unroll
        for (int e = 0; e < E; e += 2) *reinterpret_cast<float2*>(dst + lane * E + e) = make_float2(o[e], o[e + 1]);
        if (lane == 0) *reinterpret_cast<float2*>(dst + D) = make_float2(M == -INFINITY ? -INFINITY : M * kLn2, L);
    }
    // One thread waiting here for the decode grid makes this grid's completion
    // imply the decode's: a dependent's griddepcontrol.wait (before any of
    // its stores) then orders it after both.
    if (blockIdx.x == 0 && threadIdx.x == 0) ptx::grid_dependency_wait();
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

// Workspace layout: counters [B*Hkv] u32 | part_ml [slots][G][2] | part_o [slots][G][D],
// slots = (max persistent CTAs) + B*Hkv.
struct Plan {
    int max_units, slots;
    size_t cnt_off, ml_off, o_off, ws;
};

Plan make_plan(int B, int Hq, int Hkv, int D, int max_seq_len) {
    Plan pl;
    pl.max_units = (max_seq_len + 15) / 16;
    if (pl.max_units < 1) pl.max_units = 1;
    const int G = Hq / Hkv;
    pl.slots = kCtasPerSm * sm_count() + B * Hkv;
    pl.cnt_off = 0;
    pl.ml_off = align_up((size_t)B * Hkv * sizeof(unsigned long long), 256);
    pl.o_off = pl.ml_off + align_up((size_t)pl.slots * G * 2 * sizeof(float), 256);
    pl.ws = pl.o_off + align_up((size_t)pl.slots * G * D * sizeof(float), 256);
    return pl;
}

template <int D, bool BF16, int NT>
int launch_decode_t(const CUtensorMap& mk, const CUtensorMap& mv, const DecodeParams& p, cudaStream_t st) {
    auto kern = fog_decode_kernel<D, BF16, NT>;
    const int smem = Smem<D, NT>::kAlloc;
    static int occ_cache[64] = {0};
    static std::atomic<uint64_t> attr_set{0};            // bit d: the smem attribute is set on device d
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = dev < 64 ? (1ull << dev) : 0ull;
    if (!(attr_set.load(std::memory_order_acquire) & bit)) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
            return check_launch("decode: set smem attribute");
        attr_set.fetch_or(bit, std::memory_order_acq_rel);
    }
    int occ = dev < 64 ? occ_cache[dev] : 0;
    if (occ <= 0) {
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kThreads, smem) != cudaSuccess || occ <= 0)
            return set_error(KESSIE_ERR_CUDA, "paged_fog_decode: kernel does not fit on an SM");
        if (occ > kCtasPerSm) occ = kCtasPerSm;
        if (dev < 64) occ_cache[dev] = occ;
    }
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(occ * sm_count());
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, mk, mv, p);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return set_error(KESSIE_ERR_CUDA, "paged_fog_decode: %s", cudaGetErrorString(e));
    }
    return check_launch("paged_fog_decode");
}

// The combine follows the decode kernel with programmatic stream
// serialization: it may start while the decode's last CTAs still merge and
// push (every decode CTA signals launch_dependents at its last segment).  It
// reads the decode's results only as epoch-tagged words of this rank's
// exchange buffer, so one thread of it waits for the decode grid, at its end.
template <int D, bool BF16>
int launch_cp_combine_t(const CpCombineParams& a, cudaStream_t st, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((a.lay.rows + 3) / 4);
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&cfg, cp_combine_kernel<D, BF16>, a);
    if (e != cudaSuccess) return set_error(KESSIE_ERR_CUDA, "paged_fog_decode_cp combine: %s", cudaGetErrorString(e));
    return check_launch("paged_fog_decode_cp combine");
}

// Shared argument checking + parameter set-up of the decode entry points.
int prepare_decode(DecodeParams& p, Plan& pl, const void* q, int64_t q_stride_b, int64_t q_stride_h,
                   const void* k_cache, const void* v_cache, int64_t page_stride, int64_t token_stride,
                   int64_t head_stride, int num_pages, int page_size, const int32_t* block_table,
                   int64_t block_table_stride, const int32_t* seq_lens, const int32_t* kv_pos_offset,
                   const int32_t* q_positions, const int32_t* clear_start, float fog_alpha,
                   const float* fog_weights, int window_size, float sm_scale, int batch, int num_q_heads,
                   int num_kv_heads, int head_dim, int max_seq_len, int dtype, void* workspace,
                   size_t workspace_bytes) {
    if (!dtype_ok(dtype)) return set_error(KESSIE_ERR_UNSUPPORTED, "paged_fog_decode_v2: dtype %d", dtype);
    if (head_dim != 64 && head_dim != 128)
        return set_error(KESSIE_ERR_UNSUPPORTED, "paged_fog_decode_v2: head_dim %d (64/128 only)", head_dim);
    if (batch <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads)
        return set_error(KESSIE_ERR_ARG, "paged_fog_decode_v2: bad head counts Hq=%d Hkv=%d", num_q_heads, num_kv_heads);
    const int G = num_q_heads / num_kv_heads;
    if (G > 16) return set_error(KESSIE_ERR_UNSUPPORTED, "paged_fog_decode_v2: Hq/Hkv=%d > 16", G);
    if (page_size <= 0 || page_size % 16 || page_size > 256)
        return set_error(KESSIE_ERR_UNSUPPORTED, "paged_fog_decode_v2: page_size %d (multiple of 16, <= 256)", page_size);
    if (!q || !k_cache || !v_cache || !block_table || !seq_lens || num_pages <= 0 || max_seq_len < 0)
        return set_error(KESSIE_ERR_ARG, "paged_fog_decode_v2: null pointer or bad size");
    if ((q_stride_h & 1) || (q_stride_b & 1) || (reinterpret_cast<uintptr_t>(q) & 3))
        return set_error(KESSIE_ERR_ARG, "paged_fog_decode_v2: q rows must be 4-byte aligned");
    const int64_t vec = dtype == KESSIE_DTYPE_F32 ? 3 : 7;      // elements per 16 bytes, minus one
    if (((token_stride | head_stride | page_stride) & vec) || (reinterpret_cast<uintptr_t>(k_cache) & 15) ||
        (reinterpret_cast<uintptr_t>(v_cache) & 15))
        return set_error(KESSIE_ERR_ARG, "paged_fog_decode_v2: cache strides/base must be 16-byte multiples");
    pl = make_plan(batch, num_q_heads, num_kv_heads, head_dim, max_seq_len);
    if ((long long)batch * num_kv_heads * pl.max_units > (1ll << 30))
        return set_error(KESSIE_ERR_UNSUPPORTED, "paged_fog_decode_v2: B*Hkv*max_seq_len/16 above 2^30");
    if (!workspace || workspace_bytes < pl.ws || (reinterpret_cast<uintptr_t>(workspace) & 255))
        return set_error(KESSIE_ERR_WORKSPACE, "paged_fog_decode_v2: workspace %zu < %zu (or not 256-byte aligned)",
                         workspace_bytes, pl.ws);
    p = DecodeParams{};
    p.q = q; p.q_sb = q_stride_b; p.q_sh = q_stride_h;
    p.block_table = block_table; p.bt_stride = block_table_stride;
    p.seq_lens = seq_lens; p.kv_off = kv_pos_offset; p.q_pos = q_positions; p.clear_start = clear_start;
    p.fog_alpha = fog_alpha; p.fog_w = fog_weights;
    p.window = window_size;
    p.scale_log2 = sm_scale * kLog2e;
    p.B = batch; p.Hq = num_q_heads; p.Hkv = num_kv_heads; p.G = G;
    p.units_per_page = page_size / 16; p.num_pages = num_pages;
    p.max_units = pl.max_units;
    char* ws = static_cast<char*>(workspace);
    p.counters = reinterpret_cast<unsigned long long*>(ws + pl.cnt_off);
    static std::atomic<uint32_t> launch_tag{0};
    uint32_t tag = ++launch_tag;
    if (tag == 0) tag = ++launch_tag;
    p.tag = tag;
    p.part_ml = reinterpret_cast<float*>(ws + pl.ml_off);
    p.part_o = reinterpret_cast<float*>(ws + pl.o_off);
    p.status = device_status_ptr();
    p.spin_ns = kSpinNs;
    p.ws_base = workspace;
    p.ws_bytes = pl.ws;
    (void)k_cache; (void)v_cache; (void)page_stride; (void)token_stride; (void)head_stride;
    return 0;
}

int run_decode(const DecodeParams& p, const void* k_cache, const void* v_cache, int64_t page_stride,
               int64_t token_stride, int64_t head_stride, int page_size, int head_dim, bool bf16, cudaStream_t st) {
    CUtensorMap mk, mv;
    CUresult r1 = encode_kv_tile_map_cached(&mk, k_cache, bf16, head_dim, page_size, p.Hkv, p.num_pages, token_stride,
                                     head_stride, page_stride);
    CUresult r2 = encode_kv_tile_map_cached(&mv, v_cache, bf16, head_dim, page_size, p.Hkv, p.num_pages, token_stride,
                                     head_stride, page_stride);
    if (r1 != CUDA_SUCCESS || r2 != CUDA_SUCCESS)
        return set_error(KESSIE_ERR_ARG, "paged_fog_decode_v2: TMA descriptor rejected (%d/%d)", (int)r1, (int)r2);
    // Early reads when the preceding programmatic launches on the stream wrote
    // none of the inputs (with fog weights, whose extent the host does not
    // know, no).
    // After a launch that signals before its own wait (the context-parallel
    // combine) the preceding grid can run for up to its delay bound while
    // this one's warps wait in griddepcontrol.wait: the mbarrier waits get
    // that much longer.
    LaunchOrderGuard order;                  // held until the launch below is issued
    DecodeParams pe = p;
    {
        const int ps = p.units_per_page * 16;
        const int64_t kv_e = (int64_t)(p.num_pages - 1) * page_stride + (int64_t)(ps - 1) * token_stride +
                             (int64_t)(p.Hkv - 1) * head_stride + head_dim;
        const int64_t q_e = (int64_t)(p.B - 1) * p.q_sb + (int64_t)(p.Hq - 1) * p.q_sh + head_dim;
        const int64_t nb = (int64_t)p.B * 4;
        const int64_t recall_bytes = p.bias.on && p.bias.recall ? ((int64_t)p.bias.recall_nbits + 31) / 32 * 4 : 0;
        const ByteRange reads[9] = {byte_span(p.q, q_e * 2), byte_span(k_cache, kv_e * 2), byte_span(v_cache, kv_e * 2),
                                    byte_span(p.block_table, (int64_t)p.B * p.bt_stride * 4),
                                    byte_span(p.seq_lens, nb), byte_span(p.kv_off, nb), byte_span(p.q_pos, nb),
                                    byte_span(p.clear_start, nb), byte_span(p.bias.recall, recall_bytes)};
        const CpLayout lay{p.cp.world, p.B * p.Hq, head_dim};
        const ByteRange writes[4] = {byte_span(p.out, (int64_t)p.B * p.Hq * head_dim * 2),
                                     byte_span(p.out_part, (int64_t)p.B * p.Hq * (head_dim + 2) * 4),
                                     byte_span(p.ws_base, (int64_t)p.ws_bytes),
                                     byte_span(p.cp.world > 0 ? p.cp.peer[p.cp.rank] : nullptr, (int64_t)lay.bytes())};
        const bool fwd = page_stride >= 0 && token_stride >= 0 && head_stride >= 0 && p.q_sb >= 0 && p.q_sh >= 0;
        uint64_t prev_delay = 0;
        const bool ok = claim_early_reads(st, reads, 9, writes, 4, &prev_delay);
        pe.early = ok && fwd && !p.fog_w ? 1 : 0;
        if (pe.early) pe.spin_ns = prev_delay < kSpinMaxNs - kSpinNs ? kSpinNs + prev_delay : kSpinMaxNs;
    }
    const bool nt2 = p.G > 8;
    if (head_dim == 128) {
        if (bf16) return nt2 ? launch_decode_t<128, true, 2>(mk, mv, pe, st) : launch_decode_t<128, true, 1>(mk, mv, pe, st);
        return nt2 ? launch_decode_t<128, false, 2>(mk, mv, pe, st) : launch_decode_t<128, false, 1>(mk, mv, pe, st);
    }
    if (bf16) return nt2 ? launch_decode_t<64, true, 2>(mk, mv, pe, st) : launch_decode_t<64, true, 1>(mk, mv, pe, st);
    return nt2 ? launch_decode_t<64, false, 2>(mk, mv, pe, st) : launch_decode_t<64, false, 1>(mk, mv, pe, st);
}

}  // namespace
}  // namespace kessie

using namespace kessie;

extern "C" size_t kessie_paged_fog_decode_workspace_size(int batch, int num_q_heads, int num_kv_heads, int head_dim,
                                                         int max_seq_len, int page_size) {
    (void)page_size;
    if (batch <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 || num_q_heads % num_kv_heads) return 0;
    return make_plan(batch, num_q_heads, num_kv_heads, head_dim, max_seq_len).ws;
}

namespace kessie {
namespace {
int decode_entry(const void* q, int64_t q_stride_b, int64_t q_stride_h, const void* k_cache, const void* v_cache,
                 int64_t page_stride, int64_t token_stride, int64_t head_stride, int num_pages, int page_size,
                 const int32_t* block_table, int64_t block_table_stride, const int32_t* seq_lens,
                 const int32_t* kv_pos_offset, const int32_t* q_positions, const int32_t* clear_start, float fog_alpha,
                 const float* fog_weights, int window_size, float sm_scale, int batch, int num_q_heads,
                 int num_kv_heads, int head_dim, int max_seq_len, int dtype, const kessie_fog_bias* bias, void* out,
                 float* out_partial, void* workspace, size_t workspace_bytes, int phases, void* stream) {
    NvtxRange nvtx_range("kessie_paged_fog_decode");
    if (phases < 1 || phases > 3) return set_error(KESSIE_ERR_ARG, "paged_fog_decode_v2: phases %d", phases);
    DecodeParams p;
    Plan pl;
    int rc = prepare_decode(p, pl, q, q_stride_b, q_stride_h, k_cache, v_cache, page_stride, token_stride, head_stride,
                            num_pages, page_size, block_table, block_table_stride, seq_lens, kv_pos_offset,
                            q_positions, clear_start, fog_alpha, fog_weights, window_size, sm_scale, batch,
                            num_q_heads, num_kv_heads, head_dim, max_seq_len, dtype, workspace, workspace_bytes);
    if (rc) return rc;
    rc = fog_bias_from_c(bias, &p.bias);
    if (rc) return rc;
    if (!out && !out_partial) return set_error(KESSIE_ERR_ARG, "paged_fog_decode_v2: no output");
    if ((reinterpret_cast<uintptr_t>(out) & 7) || (reinterpret_cast<uintptr_t>(out_partial) & 7))
        return set_error(KESSIE_ERR_ARG, "paged_fog_decode_v2: outputs must be 8-byte aligned");
    if (dtype == KESSIE_DTYPE_F32 && p.bias.on)
        return set_error(KESSIE_ERR_UNSUPPORTED, "paged_fog_decode_v2: the additive fog bias needs f16/bf16");
    if (!(phases & 1)) { clear_error(); return 0; }      // the merge runs inside the decode kernel
    if (dtype == KESSIE_DTYPE_F32) {
        DecodeF32Args a{};
        a.q = static_cast<const float*>(q); a.q_sb = q_stride_b; a.q_sh = q_stride_h;
        a.k_cache = static_cast<const float*>(k_cache); a.v_cache = static_cast<const float*>(v_cache);
        a.page_stride = page_stride; a.token_stride = token_stride; a.head_stride = head_stride;
        a.num_pages = num_pages; a.page_size = page_size;
        a.block_table = block_table; a.bt_stride = block_table_stride;
        a.seq_lens = seq_lens; a.kv_off = kv_pos_offset; a.q_pos = q_positions; a.clear_start = clear_start;
        a.fog_alpha = fog_alpha; a.fog_w = fog_weights; a.window = window_size; a.sm_scale = sm_scale;
        a.B = batch; a.Hq = num_q_heads; a.Hkv = num_kv_heads; a.D = head_dim; a.max_seq_len = pl.max_units * 16;
        a.counters = p.counters; a.tag = p.tag; a.part_ml = p.part_ml; a.part_o = p.part_o; a.slots = pl.slots;
        a.out = static_cast<float*>(out); a.out_sb = (int64_t)num_q_heads * head_dim; a.out_sh = head_dim;
        a.out_part = out_partial; a.status = p.status;
        return launch_decode_f32(a, as_stream(stream));
    }
    p.out = out;
    p.out_part = out_partial;
    p.cp.world = 0;
    return run_decode(p, k_cache, v_cache, page_stride, token_stride, head_stride, page_size, head_dim,
                      dtype == KESSIE_DTYPE_BF16, as_stream(stream));
}
}  // namespace
}  // namespace kessie

extern "C" int kessie_paged_fog_decode_ex_v2(
    const void* q, int64_t q_stride_b, int64_t q_stride_h, const void* k_cache, const void* v_cache,
    int64_t page_stride, int64_t token_stride, int64_t head_stride, int num_pages, int page_size,
    const int32_t* block_table, int64_t block_table_stride, const int32_t* seq_lens, const int32_t* kv_pos_offset,
    const int32_t* q_positions, const int32_t* clear_start, float fog_alpha, const float* fog_weights,
    int window_size, float sm_scale, int batch, int num_q_heads, int num_kv_heads, int head_dim, int max_seq_len,
    int dtype, void* out, float* out_partial, void* workspace, size_t workspace_bytes, int phases, void* stream) {
    return decode_entry(q, q_stride_b, q_stride_h, k_cache, v_cache, page_stride, token_stride, head_stride, num_pages,
                        page_size, block_table, block_table_stride, seq_lens, kv_pos_offset, q_positions, clear_start,
                        fog_alpha, fog_weights, window_size, sm_scale, batch, num_q_heads, num_kv_heads, head_dim,
                        max_seq_len, dtype, nullptr, out, out_partial, workspace, workspace_bytes, phases, stream);
}

extern "C" int kessie_paged_fog_decode_biased_v2(
    const void* q, int64_t q_stride_b, int64_t q_stride_h, const void* k_cache, const void* v_cache,
    int64_t page_stride, int64_t token_stride, int64_t head_stride, int num_pages, int page_size,
    const int32_t* block_table, int64_t block_table_stride, const int32_t* seq_lens, const int32_t* kv_pos_offset,
    const int32_t* q_positions, const int32_t* clear_start, float fog_alpha, const float* fog_weights,
    int window_size, float sm_scale, int batch, int num_q_heads, int num_kv_heads, int head_dim, int max_seq_len,
    int dtype, const kessie_fog_bias* bias, void* out, float* out_partial, void* workspace, size_t workspace_bytes,
    void* stream) {
    return decode_entry(q, q_stride_b, q_stride_h, k_cache, v_cache, page_stride, token_stride, head_stride, num_pages,
                        page_size, block_table, block_table_stride, seq_lens, kv_pos_offset, q_positions, clear_start,
                        fog_alpha, fog_weights, window_size, sm_scale, batch, num_q_heads, num_kv_heads, head_dim,
                        max_seq_len, dtype, bias, out, out_partial, workspace, workspace_bytes, 3, stream);
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

extern "C" size_t kessie_cp_exchange_bytes(int world, int batch, int num_q_heads, int num_kv_heads, int head_dim) {
    if (world <= 0 || world > kCpMaxRanks || batch <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0)
        return 0;
    const CpLayout lay{world, batch * num_q_heads, head_dim};
    return lay.bytes();
}

namespace kessie {
namespace {
int cp_combine(void* const* exchange_buffers, int rank, int world, uint32_t epoch, int64_t wait_timeout_ns, int batch,
               int num_q_heads, int num_kv_heads, int head_dim, int dtype, void* out, float* out_partial, void* stream,
               bool follows_decode) {
    NvtxRange nvtx_range("kessie_cp_combine");
    if (world < 1 || world > kCpMaxRanks || rank < 0 || rank >= world || !exchange_buffers || !exchange_buffers[rank])
        return set_error(KESSIE_ERR_ARG, "cp_combine_v2: rank %d / world %d / buffers", rank, world);
    if (epoch == 0 || wait_timeout_ns <= 0) return set_error(KESSIE_ERR_ARG, "cp_combine_v2: epoch / timeout");
    if (dtype != KESSIE_DTYPE_BF16 && dtype != KESSIE_DTYPE_F16)
        return set_error(KESSIE_ERR_UNSUPPORTED, "cp_combine_v2: dtype %d", dtype);
    if ((head_dim != 64 && head_dim != 128) || batch <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads ||
        num_q_heads / num_kv_heads > 16)
        return set_error(KESSIE_ERR_UNSUPPORTED, "cp_combine_v2: shape");
    if (!out && !out_partial) return set_error(KESSIE_ERR_ARG, "cp_combine_v2: no output");
    if ((reinterpret_cast<uintptr_t>(out) & 7) || (reinterpret_cast<uintptr_t>(out_partial) & 7))
        return set_error(KESSIE_ERR_ARG, "cp_combine_v2: outputs must be 8-byte aligned");
    CpCombineParams a;
    a.buf = exchange_buffers[rank];
    a.lay = CpLayout{world, batch * num_q_heads, head_dim};
    a.Hq = num_q_heads;
    a.epoch = epoch; a.wait_ns = wait_timeout_ns;
    a.out = out; a.out_part = out_partial;
    a.status = device_status_ptr();
    const bool bf16 = dtype == KESSIE_DTYPE_BF16;
    cudaStream_t st = as_stream(stream);
    const bool pdl = follows_decode;
    // The combine signals its dependents at its start, before its wait for
    // the decode: its record keeps the decode's writes, and its dependents may
    // sit in griddepcontrol.wait for its cross-rank wait (plus the decode's
    // tail, bounded by the decode's own waits).
    LaunchOrderGuard order;
    const int64_t rows = (int64_t)batch * num_q_heads;
    const ByteRange writes[2] = {byte_span(out, rows * head_dim * 2), byte_span(out_partial, rows * (head_dim + 2) * 4)};
    uint64_t prev_delay = 0;
    claim_early_reads(st, nullptr, 0, writes, 2, &prev_delay, (uint64_t)wait_timeout_ns + kSpinNs, true);
    if (head_dim == 128) return bf16 ? launch_cp_combine_t<128, true>(a, st, pdl) : launch_cp_combine_t<128, false>(a, st, pdl);
    return bf16 ? launch_cp_combine_t<64, true>(a, st, pdl) : launch_cp_combine_t<64, false>(a, st, pdl);
}
}  // namespace
}  // namespace kessie

extern "C" int kessie_cp_combine_v2(void* const* exchange_buffers, int rank, int world, uint32_t epoch,
                                   int64_t wait_timeout_ns, int batch, int num_q_heads, int num_kv_heads,
                                   int head_dim, int dtype, void* out, float* out_partial, void* stream) {
    return cp_combine(exchange_buffers, rank, world, epoch, wait_timeout_ns, batch, num_q_heads, num_kv_heads,
                      head_dim, dtype, out, out_partial, stream, false);
}

extern "C" int kessie_paged_fog_decode_cp_v2(
    const void* q, int64_t q_stride_b, int64_t q_stride_h, const void* k_cache, const void* v_cache,
    int64_t page_stride, int64_t token_stride, int64_t head_stride, int num_pages, int page_size,
    const int32_t* block_table, int64_t block_table_stride, const int32_t* seq_lens, const int32_t* kv_pos_offset,
    const int32_t* q_positions, const int32_t* clear_start, float fog_alpha, const float* fog_weights,
    int window_size, float sm_scale, int batch, int num_q_heads, int num_kv_heads, int head_dim, int max_seq_len,
    int dtype, void* const* exchange_buffers, int rank, int world, uint32_t epoch, int64_t wait_timeout_ns,
    void* out, float* out_partial, void* workspace, size_t workspace_bytes, int phases, void* stream) {
    if (phases < 1 || phases > 3) return set_error(KESSIE_ERR_ARG, "paged_fog_decode_cp_v2: phases %d", phases);
    if (world < 1 || world > kCpMaxRanks || rank < 0 || rank >= world)
        return set_error(KESSIE_ERR_ARG, "paged_fog_decode_cp_v2: rank %d / world %d (1..%d ranks)", rank, world,
                         kCpMaxRanks);
    if (epoch == 0) return set_error(KESSIE_ERR_ARG, "paged_fog_decode_cp_v2: epoch must be non-zero");
    if (wait_timeout_ns <= 0) return set_error(KESSIE_ERR_ARG, "paged_fog_decode_cp_v2: wait_timeout_ns must be > 0");
    if (!exchange_buffers) return set_error(KESSIE_ERR_ARG, "paged_fog_decode_cp_v2: null exchange_buffers");
    for (int r = 0; r < world; ++r)
        if (!exchange_buffers[r] || (reinterpret_cast<uintptr_t>(exchange_buffers[r]) & 255))
            return set_error(KESSIE_ERR_ARG, "paged_fog_decode_cp_v2: exchange buffer %d null or not 256-byte aligned", r);
    if ((phases & 2) && !out && !out_partial) return set_error(KESSIE_ERR_ARG, "paged_fog_decode_cp_v2: no output");
    if (dtype == KESSIE_DTYPE_F32)
        return set_error(KESSIE_ERR_UNSUPPORTED, "paged_fog_decode_cp_v2: dtype f32 (f16/bf16 only)");
    DecodeParams p;
    Plan pl;
    int rc = prepare_decode(p, pl, q, q_stride_b, q_stride_h, k_cache, v_cache, page_stride, token_stride, head_stride,
                            num_pages, page_size, block_table, block_table_stride, seq_lens, kv_pos_offset,
                            q_positions, clear_start, fog_alpha, fog_weights, window_size, sm_scale, batch,
                            num_q_heads, num_kv_heads, head_dim, max_seq_len, dtype, workspace, workspace_bytes);
    if (rc) return rc;
    const bool bf16 = dtype == KESSIE_DTYPE_BF16;
    cudaStream_t st = as_stream(stream);
    if (phases & 1) {
        p.out = nullptr;
        p.out_part = nullptr;
        for (int r = 0; r < kCpMaxRanks; ++r) p.cp.peer[r] = r < world ? exchange_buffers[r] : nullptr;
        p.cp.rank = rank; p.cp.world = world; p.cp.epoch = epoch;
        rc = run_decode(p, k_cache, v_cache, page_stride, token_stride, head_stride, page_size, head_dim, bf16, st);
        if (rc) return rc;
    }
    if (phases & 2) {
        rc = cp_combine(exchange_buffers, rank, world, epoch, wait_timeout_ns, batch, num_q_heads, num_kv_heads,
                        head_dim, dtype, out, out_partial, stream, (phases & 1) != 0);
        if (rc) return rc;
    }
    clear_error();
    return 0;
}

extern "C" int kessie_lse_combine_v2(const float* partials, int num_splits, int64_t split_stride, int rows,
                                     int head_dim, void* out, int out_dtype, float* out_partial, void* stream) {
    NvtxRange nvtx_range("kessie_lse_combine_v2");
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
// cached; make that first call before any stream capture.  The cache is never
// refreshed: after cudaDeviceReset (or anything else that tears down the
// device's primary context) the cached address is stale, so a process that
// resets a device must not call this entry point on it again.  All calls share
// the one array, so two calls whose work overlaps on the GPU (different
// streams, or different threads using one device) race on it; callers must
// order them.  The array keeps whatever the previous call left: the decode's
// per-group arrival counters carry a per-launch tag (a stale tag counts as
// zero), and every partial the decode reads it has written in the same call.
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
        if (e != cudaSuccess || !p) {
            cudaGetLastError();       // consume the error so a later call's launch check does not see it
            return set_error(KESSIE_ERR_CUDA, "noalloc decode: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
        }
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
    NvtxRange nvtx_range("kessie_paged_fog_decode_noalloc_v2");
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
