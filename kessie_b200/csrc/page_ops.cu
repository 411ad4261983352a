// page_ops.cu -- RoPE remap, page evict/compaction, page insert(+remap), page gather.
//
// All four are HBM-bound byte movers.  Layout rules:
//   * head_dim is contiguous; every row moves as 16-byte vectors
//     (8 x fp16/bf16 or 4 x fp32), one vector per thread per token.
//   * a CTA owns one page (insert / gather) or a group of tokens (remap) and
//     loops over its tokens with the loads issued back to back, so each
//     thread keeps page_size 16-byte loads in flight with no index math in the
//     loop body.
//   * the RoPE angle depends on (token, d) only, so cos/sin are computed once
//     per token into shared memory and reused by every head.
// Semantics follow kessie_kernels_v2.hip:393-456,670-707 and
// kessie_hip_kernels.py:520-564,596-606 (see each kernel).
#include "common.cuh"
#include "ptx.cuh"

#include <math.h>
#include <stdio.h>

#include <algorithm>

namespace kessie {
namespace {

constexpr int kMaxHalf = 128;   // head_dim <= 256

struct FreqTable { float f[kMaxHalf]; };

// 1/theta^(d/half): theta^e in float64 rounded to fp32, then the fp32
// reciprocal -- the two roundings of the reference's torch expression
// (kessie_hip_kernels.py:600) with a correctly rounded pow.
FreqTable make_freqs(float theta, int half) {
    FreqTable t;
    for (int d = 0; d < kMaxHalf; ++d) {
        if (d < half) {
            float e = (float)d / (float)half;
            float p = (float)pow((double)theta, (double)e);
            t.f[d] = 1.0f / p;
        } else {
            t.f[d] = 0.f;
        }
    }
    return t;
}

// cos / sin of the reference's fp32 angle x = (float)(tgt - orig) * f_d.
// |x| reaches ~1.6e5 rad, where the accurate sincosf takes its slow
// large-argument path (and diverges across the lanes of a warp).  x itself is
// kept bit-for-bit (it carries the reference's fp32 rounding); it is reduced
// to [-pi, pi] in double precision -- exact to ~1e-11 rad at these magnitudes
// -- and evaluated with the hardware approximation (abs error < 4e-7).
__device__ __forceinline__ void rope_sincos(float x, float* s, float* c) {
    const double xd = (double)x;
    const double k = rint(xd * 0.15915494309189535);          // 1 / (2 pi)
    const float r = (float)fma(-k, 6.283185307179586, xd);    // x - 2 pi k
    __sincosf(r, s, c);
}

// ------------------------------------------------------------------ vectors
template <typename T> struct VecOps;
template <> struct VecOps<__half> {
    static constexpr int N = 8;
    __device__ static void unpack(uint4 v, float* f) {
        const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
        for (int i = 0; i < 4; ++i) { float2 x = __half22float2(h[i]); f[2 * i] = x.x; f[2 * i + 1] = x.y; }
    }
    __device__ static uint4 pack(const float* f) {
        uint4 v; __half2* h = reinterpret_cast<__half2*>(&v);
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
        return v;
    }
};
template <> struct VecOps<__nv_bfloat16> {
    static constexpr int N = 8;
    __device__ static void unpack(uint4 v, float* f) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
        for (int i = 0; i < 4; ++i) { float2 x = __bfloat1622float2(h[i]); f[2 * i] = x.x; f[2 * i + 1] = x.y; }
    }
    __device__ static uint4 pack(const float* f) {
        uint4 v; __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
        return v;
    }
};
template <> struct VecOps<float> {
    static constexpr int N = 4;
    __device__ static void unpack(uint4 v, float* f) { f[0] = __uint_as_float(v.x); f[1] = __uint_as_float(v.y); f[2] = __uint_as_float(v.z); f[3] = __uint_as_float(v.w); }
    __device__ static uint4 pack(const float* f) { return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3])); }
};

// Rotate one (lo, hi) pair of 16-byte vectors: lo' = lo c - hi s, hi' = lo s + hi c
// (kessie_kernels_v2.hip:697-706; fp32 math, round once to storage).
template <typename T>
__device__ __forceinline__ void rotate_pair(uint4& lo, uint4& hi, const float* c, const float* s) {
    constexpr int N = VecOps<T>::N;
    float a[N], b[N], ra[N], rb[N];
    VecOps<T>::unpack(lo, a);
    VecOps<T>::unpack(hi, b);
#pragma unroll
    for (int i = 0; i < N; ++i) {
        ra[i] = a[i] * c[i] - b[i] * s[i];
        rb[i] = a[i] * s[i] + b[i] * c[i];
    }
    lo = VecOps<T>::pack(ra);
    hi = VecOps<T>::pack(rb);
}

// ------------------------------------------------------------------ bulk-copy page gather
// Persistent, warp-specialised CTAs (one per SM) gather pages with the
// bulk-copy (TMA) engine instead of through registers.  A unit is one
// gathered page: its K rows and V rows (a row = all heads of one token, H*D
// contiguous elements; 2 x 16 x 2 KB = 64 KB at config 2).  A ring of
// shared-memory stages carries the units:
//   warp 0 (producer): one global->shared bulk load per row of unit k into
//           stage k % ns once the stage is released (empty[s]); completion on
//           full[s];
//   warp 1 (storer): waits for full[s], issues one shared->global bulk store
//           per output row (row-sized copies measured faster than one 32 KB
//           copy per block), and releases a stage once the
//           stores that read it are done (bulk-group read wait, one unit
//           behind).
// Sources and destinations are this GPU's memory; no multicast.  Every wait
// is bounded; a wait that runs out flags KESSIE_DEV_WAIT_TIMEOUT, stops both
// roles, and the CTA lets its issued copies finish before exiting.
constexpr int kBulkMaxStages = 8;
constexpr int kBulkStoreLag = 1;       // store groups left in flight before a stage is released
constexpr int kBulkHeader = 256;       // barriers and the abort flag

struct BulkArgs {
    const char* cache;              // source pages
    int64_t page_b, token_b, kv_b;  // byte strides of the cache
    int max_pages, ps;
    const int32_t* ids;             // page of unit i
    char* rk;                       // dense K output rows [n*ps][H][D] (nullable)
    char* rv;                       // dense V output rows (nullable)
    int R;                          // bytes of one row (H*D elements), a multiple of 16
    int units;
    int ns, stage_b;                // ring stages, bytes per stage
    int* status;
    int early;                      // first ring fill before griddepcontrol.wait
};

__global__ void __launch_bounds__(64, 1) page_gather_bulk_kernel(const BulkArgs a) {
    extern __shared__ __align__(128) uint8_t bsm[];
    uint64_t* full = reinterpret_cast<uint64_t*>(bsm);                 // [ns]
    uint64_t* empty = full + kBulkMaxStages;                           // [ns]
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bsm + 2 * kBulkMaxStages * 8);
    uint8_t* stages = bsm + kBulkHeader;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int my_units = a.units > (int)blockIdx.x ? (a.units - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    auto unit_of = [&](int k) { return (int)blockIdx.x + k * (int)gridDim.x; };
    auto page_of = [&](int u) -> int {
        const int pg = a.ids[u];
        return (pg < 0 || pg >= a.max_pages) ? -1 : pg;
    };
    if (threadIdx.x == 0) {
        for (int s = 0; s < a.ns; ++s) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], 1);
        }
        *abort_flag = 0;
        ptx::fence_mbar_init();
    }
    __syncthreads();
    // Programmatic dependent launch: a thread touches global memory only after
    // the preceding grid has completed (griddepcontrol.wait), then lets the
    // next launch start.  With a.early the producer issues its first ring
    // fill (reads of the page ids and of the cache only) before its wait; the
    // host allows that only when the preceding programmatic launch of this
    // library wrote none of those bytes.  Every store follows the wait.
    const bool early_producer = a.early && threadIdx.x == 0;
    if (!early_producer) {
        ptx::grid_dependency_wait();
        ptx::launch_dependents();
    }
    const uint32_t R = (uint32_t)a.R;
    const uint32_t blk = (uint32_t)a.ps * R;          // one K (or V) block of a page
    auto fail = [&]() {
        record_status(a.status, KESSIE_DEV_WAIT_TIMEOUT);
        *abort_flag = 1;
    };
    if (warp == 0) {
        // ------------------------------------------------------------ producer
        int issued = 0;
        if (lane == 0) {
            bool waited = !early_producer;
            for (int k = 0; k < my_units && !*abort_flag; ++k) {
                if (!waited && k == a.ns) {
                    ptx::grid_dependency_wait();
                    waited = true;
                }
                const int s = k % a.ns;
                if (k >= a.ns && !ptx::mbar_wait(&empty[s], (uint32_t)(k / a.ns - 1) & 1u)) { fail(); break; }
                const int pg = page_of(unit_of(k));
                uint8_t* st = stages + (size_t)s * a.stage_b;
                const int nb = pg < 0 ? 0 : (a.rk ? 1 : 0) + (a.rv ? 1 : 0);
                ptx::mbar_arrive_expect_tx(&full[s], (uint32_t)nb * blk);
                if (pg >= 0) {
                    const char* page = a.cache + (int64_t)pg * a.page_b;
                    for (int b = 0; b < 2; ++b) {
                        if (!(b ? a.rv : a.rk)) continue;
                        for (int t = 0; t < a.ps; ++t)
                            ptx::bulk_g2s(st + b * blk + t * R, page + t * a.token_b + b * a.kv_b, R, &full[s]);
                    }
                }
                issued = k + 1;
            }
            if (!waited) ptx::grid_dependency_wait();
        }
        __syncwarp();
        // the CTA exits only after every issued load has landed (bounded)
        if (lane == 0)
            for (int k = max(0, issued - a.ns); k < issued; ++k)
                if (!ptx::mbar_wait(&full[k % a.ns], (uint32_t)(k / a.ns) & 1u)) { fail(); break; }
    } else {
        // ------------------------------------------------------------ storer
        for (int k = 0; k < my_units; ++k) {
            if (__any_sync(0xffffffffu, *abort_flag != 0)) break;
            const int s = k % a.ns;
            if (!__all_sync(0xffffffffu, ptx::mbar_wait(&full[s], (uint32_t)(k / a.ns) & 1u))) {
                if (lane == 0) fail();
                break;
            }
            const int u = unit_of(k);
            const int pg = page_of(u);
            const uint8_t* st = stages + (size_t)s * a.stage_b;
            const int64_t off = (int64_t)u * blk;     // dense output rows of this page
            if (pg < 0) {
                // a bad page id gathers zeros
                if (lane == 0) record_status(a.status, KESSIE_DEV_BAD_PAGE_ID);
                for (int b = 0; b < 2; ++b) {
                    char* out = b ? a.rv : a.rk;
                    if (!out) continue;
                    for (uint32_t i = lane * 16; i < blk; i += 32 * 16)
                        *reinterpret_cast<uint4*>(out + off + i) = make_uint4(0, 0, 0, 0);
                }
            } else if (lane == 0) {
                for (int b = 0; b < 2; ++b) {
                    char* out = b ? a.rv : a.rk;
                    if (!out) continue;
                    for (int t = 0; t < a.ps; ++t) ptx::bulk_s2g(out + off + t * R, st + b * blk + t * R, R);
                }
            }
            if (lane == 0) {
                ptx::bulk_commit();
                ptx::bulk_wait_read<kBulkStoreLag>();
                if (k >= kBulkStoreLag) ptx::mbar_arrive(&empty[(k - kBulkStoreLag) % a.ns]);
            }
            __syncwarp();
        }
        if (lane == 0) ptx::bulk_wait<0>();
    }
    __syncthreads();
}

// Bulk gather set-up: rows of H*D contiguous elements (head stride ==
// head_dim), 16-byte aligned bases and strides, dense outputs, and a ring of
// >= 3 stages in shared memory.  Returns 0 when the shape is outside it.
int launch_gather_bulk(BulkArgs a, cudaStream_t st) {
    const int budget = 227 * 1024;
    a.stage_b = (int)align_up((size_t)2 * a.ps * a.R, 128);
    a.ns = std::min(kBulkMaxStages, (budget - kBulkHeader) / a.stage_b);
    if (a.ns < kBulkStoreLag + 2) return 0;
    const int smem = kBulkHeader + a.ns * a.stage_b;
    if (cudaFuncSetAttribute(page_gather_bulk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
        cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    const int grid = std::min(a.units, sm_count());
    LaunchOrderGuard order;                  // held until the launch below is issued
    // early reads: the cache rows and page ids this gather reads against the
    // bytes the preceding programmatic launch on the stream wrote
    {
        const uintptr_t cb = reinterpret_cast<uintptr_t>(a.cache), ib = reinterpret_cast<uintptr_t>(a.ids);
        const int64_t span = (int64_t)(a.max_pages - 1) * a.page_b + (int64_t)(a.ps - 1) * a.token_b +
                             (a.rv ? a.kv_b : 0) + a.R;
        const bool fwd = a.page_b >= 0 && a.token_b >= 0 && a.kv_b >= 0;
        const ByteRange reads[2] = {{cb, cb + (uintptr_t)span}, {ib, ib + (uintptr_t)a.units * 4}};
        const uintptr_t kb = reinterpret_cast<uintptr_t>(a.rk), vb = reinterpret_cast<uintptr_t>(a.rv);
        const uintptr_t out_b = (uintptr_t)a.units * a.ps * (uintptr_t)a.R;
        const ByteRange writes[2] = {a.rk ? ByteRange{kb, kb + out_b} : ByteRange{0, 0},
                                     a.rv ? ByteRange{vb, vb + out_b} : ByteRange{0, 0}};
        a.early = claim_early_reads(st, reads, 2, writes, 2) && fwd ? 1 : 0;
    }
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(64);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, page_gather_bulk_kernel, a) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return 1;
}

bool bulk_ok(int64_t bytes) { return bytes % 16 == 0; }


// Launch as a programmatic dependent of the preceding kernel on the stream.
template <typename... Params, typename... Args>
cudaError_t launch_pdl(void (*kern)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

// ------------------------------------------------------------------ RoPE remap
// CTA = `tpb` tokens.  Stage 1: cos/sin of (tgt-orig)*f_d for the CTA's tokens
// into smem.  Stage 2: every (token, head, 16B chunk of the low half) item
// loads its low/high vectors, rotates, stores.
template <typename T>
__global__ void __launch_bounds__(256) rope_remap_kernel(
    T* __restrict__ k, int num_tokens, int num_heads, int half, int64_t tstride, int64_t hstride,
    const int32_t* __restrict__ orig, const int32_t* __restrict__ tgt, FreqTable ft, int tpb) {
    extern __shared__ float sm[];
    float* cs = sm;                       // [tpb][half]
    float* sn = sm + tpb * half;          // [tpb][half]
    const int t0 = blockIdx.x * tpb;
    const int nt = min(tpb, num_tokens - t0);
    for (int i = threadIdx.x; i < nt * half; i += blockDim.x) {
        int tl = i / half, d = i - tl * half;
        int t = t0 + tl;
        float delta = (float)(tgt[t] - orig[t]) * ft.f[d];
        float s, c;
        rope_sincos(delta, &s, &c);
        cs[i] = c; sn[i] = s;
    }
    __syncthreads();
    constexpr int N = VecOps<T>::N;
    const int chunks = half / N;
    const int items = nt * num_heads * chunks;
    for (int i = threadIdx.x; i < items; i += blockDim.x) {
        int c = i % chunks;
        int r = i / chunks;
        int h = r % num_heads;
        int tl = r / num_heads;
        T* row = k + (int64_t)(t0 + tl) * tstride + (int64_t)h * hstride;
        uint4* plo = reinterpret_cast<uint4*>(row + c * N);
        uint4* phi = reinterpret_cast<uint4*>(row + half + c * N);
        uint4 lo = *plo, hi = *phi;
        rotate_pair<T>(lo, hi, cs + tl * half + c * N, sn + tl * half + c * N);
        *plo = lo; *phi = hi;
    }
}

// Element-wise variant for rows whose halves are not 16-byte aligned.
template <typename T>
__global__ void rope_remap_scalar_kernel(T* __restrict__ k, int num_tokens, int num_heads, int half,
                                         int64_t tstride, int64_t hstride, const int32_t* __restrict__ orig,
                                         const int32_t* __restrict__ tgt, FreqTable ft) {
    int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int64_t total = (int64_t)num_tokens * num_heads * half;
    if (gid >= total) return;
    int d = (int)(gid % half);
    int64_t r = gid / half;
    int h = (int)(r % num_heads);
    int t = (int)(r / num_heads);
    float delta = (float)(tgt[t] - orig[t]) * ft.f[d];
    float s, c;
    rope_sincos(delta, &s, &c);
    T* row = k + (int64_t)t * tstride + (int64_t)h * hstride;
    float a = to_f32(row[d]), b = to_f32(row[d + half]);
    row[d] = from_f32<T>(a * c - b * s);
    row[d + half] = from_f32<T>(a * s + b * c);
}


// Row-parallel rotation for the common shapes (16-byte chunks per row CPR is a
// power of two <= 32, so a row's chunks sit in aligned lanes of one warp).
// Thread = one 16-byte chunk c of one head row; it loops over the block's
// tokens with every load issued before any trig, then pairs its chunk with
// the partner half (lane ^ CPR/2) by shuffles and writes only its own half:
//   low  lanes: lo' = lo*cos - hi*sin      high lanes: hi' = lo*sin + hi*cos
// MODE 0: in place on K.  MODE 1: page insert -- K rows rotated (when
// `orig` is given) and V rows copied into page `page_ids[blockIdx.x]`.
template <typename T, int MODE, int KT>
__global__ void __launch_bounds__(256) rope_rows_kernel(
    T* __restrict__ dst, const T* __restrict__ src, const T* __restrict__ srcv, int num_tokens, int num_heads,
    int half, int cpr, int64_t src_ts, int64_t src_hs, int64_t dst_ts, int64_t dst_hs, int64_t dst_kv,
    int64_t page_stride, int page_size, const int32_t* __restrict__ page_ids, int max_pages,
    int8_t* __restrict__ valid, int32_t* __restrict__ positions, int conv_pos,
    const int32_t* __restrict__ orig, const int32_t* __restrict__ tgt, FreqTable ft, int tt, int* status) {
    extern __shared__ float sm[];
    constexpr int N = VecOps<T>::N;
    const int ipt = num_heads * cpr;                  // items per token
    const int tp = blockDim.x / ipt;                  // tokens processed in parallel
    const int tg = threadIdx.x / ipt, item = threadIdx.x - tg * ipt;
    const int h = item / cpr, c = item - h * cpr;
    const int t0 = blockIdx.x * tt;
    const int nt = min(tt, num_tokens - t0);
    T* base = dst;
    if (MODE == 1) {
        const int phys = page_ids[blockIdx.x];
        if (phys < 0 || phys >= max_pages) {
            if (threadIdx.x == 0) record_status(status, KESSIE_DEV_BAD_PAGE_ID);
            return;
        }
        if (threadIdx.x == 0 && valid) valid[phys] = 1;
        if (threadIdx.x == 0 && positions) positions[phys] = conv_pos + t0;
        base = dst + (int64_t)phys * page_stride;
    }
    // 1. loads (K rows, and V rows for the insert)
    uint4 kv[KT], vv[KT];
#pragma unroll
    for (int k = 0; k < KT; ++k) {
        const int tl = tg + tp * k;
        if (tl < nt) {
            kv[k] = ldg_stream(src + (int64_t)(t0 + tl) * src_ts + (int64_t)h * src_hs + c * N);
            if (MODE == 1) vv[k] = ldg_stream(srcv + (int64_t)(t0 + tl) * src_ts + (int64_t)h * src_hs + c * N);
        }
    }
    // 2. cos/sin per (token, d) for the block's tokens, while the loads fly
    const bool rot = orig != nullptr;
    float* cs = sm;
    float* sn = sm + tt * half;
    if (rot) {
        for (int i = threadIdx.x; i < nt * half; i += blockDim.x) {
            const int tl = i / half, d = i - tl * half;
            const int t = t0 + tl;
            const int target = tgt ? tgt[t] : conv_pos + t;
            float sv, cv;
            rope_sincos((float)(target - orig[t]) * ft.f[d], &sv, &cv);
            cs[i] = cv; sn[i] = sv;
        }
    }
    __syncthreads();
    // 3. rotate with the partner half and store
    const int hc = cpr >> 1;
    const bool lo_lane = c < hc;
    const int dbase = (lo_lane ? c : c - hc) * N;
#pragma unroll
    for (int k = 0; k < KT; ++k) {
        const int tl = tg + tp * k;
        uint4 o = kv[k];
        if (rot) {
            uint4 pr;
            pr.x = __shfl_xor_sync(0xffffffffu, kv[k].x, hc);
            pr.y = __shfl_xor_sync(0xffffffffu, kv[k].y, hc);
            pr.z = __shfl_xor_sync(0xffffffffu, kv[k].z, hc);
            pr.w = __shfl_xor_sync(0xffffffffu, kv[k].w, hc);
            if (tl < nt) {
                float a[N], b[N], r[N];
                const float* cc = cs + tl * half + dbase;
                const float* ss = sn + tl * half + dbase;
                if (lo_lane) {
                    VecOps<T>::unpack(kv[k], a); VecOps<T>::unpack(pr, b);
#pragma unroll
                    for (int i = 0; i < N; ++i) r[i] = a[i] * cc[i] - b[i] * ss[i];
                } else {
                    VecOps<T>::unpack(pr, a); VecOps<T>::unpack(kv[k], b);
#pragma unroll
                    for (int i = 0; i < N; ++i) r[i] = a[i] * ss[i] + b[i] * cc[i];
                }
                o = VecOps<T>::pack(r);
            }
        }
        if (tl < nt) {
            T* drow = base + (int64_t)(MODE == 1 ? tl : t0 + tl) * dst_ts + (int64_t)h * dst_hs + c * N;
            if (MODE == 1) {
                stg_stream(drow, o);
                stg_stream(drow + dst_kv, vv[k]);
            } else {
                *reinterpret_cast<uint4*>(drow) = o;
            }
        }
    }
}

// Launch shape of rope_rows_kernel, or false when the shape needs the generic kernels.
template <typename T>
bool rows_shape(int H, int D, int tt, int& threads, int& cpr, int& kt) {
    constexpr int N = VecOps<T>::N;
    if (D % (2 * N)) return false;
    cpr = D / N;
    if (cpr > 32 || (cpr & (cpr - 1))) return false;
    const int ipt = H * cpr;
    if (ipt > 256) return false;
    const int tp = 256 / ipt;
    threads = ipt * tp;
    if (threads % 32) return false;
    kt = (tt + tp - 1) / tp;
    return kt == 1 || kt == 2 || kt == 4 || kt == 8 || kt == 16;
}

template <typename T, int MODE>
void launch_rows(int kt, dim3 grid, int threads, size_t smem, cudaStream_t st, T* dst, const T* src, const T* srcv,
                 int T_, int H, int half, int cpr, int64_t sts, int64_t shs, int64_t dts, int64_t dhs, int64_t dkv,
                 int64_t pstride, int ps, const int32_t* ids, int maxp, int8_t* valid, int32_t* pos, int conv,
                 const int32_t* orig, const int32_t* tgt, const FreqTable& ft, int tt, int* status) {
#define KESSIE_ROWS(KT_) rope_rows_kernel<T, MODE, KT_><<<grid, threads, smem, st>>>(dst, src, srcv, T_, H, half, cpr, sts, shs, dts, dhs, dkv, pstride, ps, ids, maxp, valid, pos, conv, orig, tgt, ft, tt, status)
    switch (kt) {
        case 1: KESSIE_ROWS(1); break;
        case 2: KESSIE_ROWS(2); break;
        case 4: KESSIE_ROWS(4); break;
        case 8: KESSIE_ROWS(8); break;
        default: KESSIE_ROWS(16); break;
    }
#undef KESSIE_ROWS
}


// Token-block RoPE kernel shared by the in-place remap and the fused recall
// insert.  A CTA owns `tpb` tokens.  A thread's item is (token, head group g,
// 16-byte chunk kc of the low half); it rotates chunk kc of the HPT heads
// g, g + H/HPT, ..., so every (cos, sin) table entry it reads from shared
// memory serves HPT heads.  Order: start 16-byte cp.async copies of the
// CTA's K rows (and V rows for the insert) into shared memory -- the bytes in
// flight cost no registers, so 8 CTAs fit per SM and keep ~128 KB per SM in
// flight while each CTA builds its float4 table (cos d, sin d, cos d+1,
// sin d+1); then wait, barrier, rotate out of shared memory and store.
// INSERT: destination row of token t is page page_ids[t / ps], slot t % ps
// (first token of a page sets page_valid / page_positions); the V rows are
// copied alongside.  With bulk_st (destination rows of H*D contiguous
// elements) the insert writes its rotated K rows back into shared memory and
// every K and V row leaves as one shared->global bulk copy.
template <typename T, bool INSERT, int HPT>
__global__ void __launch_bounds__(256, INSERT ? 5 : 6) rope_tokens_kernel(
    T* __restrict__ dst, const T* __restrict__ srck, const T* __restrict__ srcv, int num_tokens, int num_heads,
    int half, int64_t sts, int64_t shs, int64_t dts, int64_t dhs, int64_t dkv, int64_t page_stride, int ps,
    const int32_t* __restrict__ page_ids, int max_pages, int8_t* __restrict__ valid, int32_t* __restrict__ positions,
    int conv_pos, const int32_t* __restrict__ orig, const int32_t* __restrict__ tgt, FreqTable ft, int tpb,
    int* status, int bulk_st, int early) {
    extern __shared__ float4 tab[];                 // [tpb][half/2] of (cos d, sin d, cos d+1, sin d+1)
    // Programmatic dependent launch: every global access follows the wait for
    // the preceding grid, then the next launch may start -- except that with
    // `early` (the host found that the preceding programmatic launch of this
    // library wrote none of the rows, positions and page ids read here) the
    // copies in and the angle table run before the wait, overlapping the
    // preceding grid's last CTAs; every store still follows it.
    if (!early) {
        ptx::grid_dependency_wait();
        ptx::launch_dependents();
    }
    constexpr int N = VecOps<T>::N;
    const int hc = half / N;                        // 16-byte chunks per half row
    const int hg = num_heads / HPT;                 // head groups
    const int rowe = num_heads * 2 * half;          // elements of one token's K (or V) row
    T* ksm = reinterpret_cast<T*>(tab + tpb * (half / 2));   // [tpb][H][D] K rows
    T* vsm = ksm + tpb * rowe;                               // [tpb][H][D] V rows (insert)
    long long* rowoff = reinterpret_cast<long long*>(vsm + (INSERT ? tpb * rowe : 0));  // [tpb] insert dst offsets
    float* fqs = reinterpret_cast<float*>(rowoff + (INSERT ? tpb : 0));                // [half] frequencies
    const int t0 = blockIdx.x * tpb;
    const int nt = min(tpb, num_tokens - t0);
    const int kitems = nt * hg * hc;                // <= blockDim by construction of tpb
    const int vitems = INSERT ? nt * num_heads * 2 * hc : 0;
    const bool kact = (int)threadIdx.x < kitems;
    int kc = 0, g = 0, ktl = 0;
    if (kact) {
        kc = threadIdx.x % hc;
        const int r = threadIdx.x / hc;
        g = r % hg;
        ktl = r / hg;
    }
    // ---- 1. async copies: HPT K pairs and (insert) 2*HPT V vectors per thread
    if (kact) {
#pragma unroll
        for (int j = 0; j < HPT; ++j) {
            const int h = g + j * hg;
            const T* row = srck + (int64_t)(t0 + ktl) * sts + (int64_t)h * shs;
            T* srow = ksm + ktl * rowe + h * 2 * half;
            cp_async16(srow + kc * N, row + kc * N);
            cp_async16(srow + half + kc * N, row + half + kc * N);
        }
    }
    if (INSERT) {
#pragma unroll
        for (int j = 0; j < 2 * HPT; ++j) {
            const int vi = threadIdx.x + j * blockDim.x;
            if (vi < vitems) {
                const int c = vi % (2 * hc), r = vi / (2 * hc);
                const int h = r % num_heads, tl = r / num_heads;
                cp_async16(vsm + tl * rowe + h * 2 * half + c * N,
                           srcv + (int64_t)(t0 + tl) * sts + (int64_t)h * shs + c * N);
            }
        }
    }
    cp_async_commit();
    // ---- 2. angle table (one float4 = two consecutive d).  The frequencies
    // go through shared memory first: a kernel parameter read at a per-thread
    // index is serialised by the constant cache.
    for (int i = threadIdx.x; i < half; i += blockDim.x) fqs[i] = ft.f[i];
    // tokens whose position moves by the same amount share one table row: a
    // recalled page moves its consecutive positions by one delta, so the
    // usual CTA (its tokens in one page) builds a single row
    auto delta = [&](int t) -> int { return (tgt ? tgt[t] : conv_pos + t) - orig[t]; };
    const int d0 = delta(t0);
    const bool uni = __syncthreads_and((int)threadIdx.x >= nt || delta(t0 + (int)threadIdx.x) == d0) != 0;
    const int hp = half / 2;
    for (int i = threadIdx.x; i < (uni ? 1 : nt) * hp; i += blockDim.x) {
        const int tl = i / hp, dp = i - tl * hp;
        const float dlt = (float)(uni ? d0 : delta(t0 + tl));
        float4 cs;
        rope_sincos(dlt * fqs[2 * dp], &cs.y, &cs.x);
        rope_sincos(dlt * fqs[2 * dp + 1], &cs.w, &cs.z);
        tab[i] = cs;
    }
    if (INSERT) {
        // destination row of each token (page, slot), once per token; the first
        // token of a page sets page_valid / page_positions
        for (int tl = threadIdx.x; tl < nt; tl += blockDim.x) {
            const int t = t0 + tl;
            const int phys = page_ids[t / ps];
            const bool ok = phys >= 0 && phys < max_pages;
            rowoff[tl] = ok ? (long long)phys * page_stride + (long long)(t % ps) * dts : -1ll;
        }
    }
    cp_async_wait_all();
    __syncthreads();
    if (early) {
        ptx::grid_dependency_wait();
        ptx::launch_dependents();
    }
    if (INSERT) {
        for (int tl = threadIdx.x; tl < nt; tl += blockDim.x) {
            const int t = t0 + tl;
            if (t % ps) continue;
            const long long off = rowoff[tl];
            if (off < 0) record_status(status, KESSIE_DEV_BAD_PAGE_ID);
            else {
                const int phys = page_ids[t / ps];
                if (valid) valid[phys] = 1;
                if (positions) positions[phys] = conv_pos + t;
            }
        }
    }
    // ---- 3. rotate the K pairs with one table read for all HPT heads; copy V
    auto dst_row = [&](int tl, int h, bool& ok) -> T* {
        if (!INSERT) { ok = true; return dst + (int64_t)(t0 + tl) * dts + (int64_t)h * dhs; }
        const long long off = rowoff[tl];
        ok = off >= 0;
        return dst + (ok ? off : 0) + (int64_t)h * dhs;
    };
    if (kact) {
        float4 cs[N / 2];
        const float4* tp = tab + (uni ? 0 : ktl * hp) + kc * (N / 2);
#pragma unroll
        for (int q = 0; q < N / 2; ++q) cs[q] = tp[q];
#pragma unroll
        for (int j = 0; j < HPT; ++j) {
            float a[N], bb[N], ra[N], rb[N];
            const T* srow = ksm + ktl * rowe + (g + j * hg) * 2 * half;
            VecOps<T>::unpack(*reinterpret_cast<const uint4*>(srow + kc * N), a);
            VecOps<T>::unpack(*reinterpret_cast<const uint4*>(srow + half + kc * N), bb);
#pragma unroll
            for (int q = 0; q < N / 2; ++q) {
                ra[2 * q] = a[2 * q] * cs[q].x - bb[2 * q] * cs[q].y;
                rb[2 * q] = a[2 * q] * cs[q].y + bb[2 * q] * cs[q].x;
                ra[2 * q + 1] = a[2 * q + 1] * cs[q].z - bb[2 * q + 1] * cs[q].w;
                rb[2 * q + 1] = a[2 * q + 1] * cs[q].w + bb[2 * q + 1] * cs[q].z;
            }
            if (INSERT && bulk_st) {
                // rotated in place; the rows leave through the bulk-copy engine below
                T* wrow = ksm + ktl * rowe + (g + j * hg) * 2 * half;
                *reinterpret_cast<uint4*>(wrow + kc * N) = VecOps<T>::pack(ra);
                *reinterpret_cast<uint4*>(wrow + half + kc * N) = VecOps<T>::pack(rb);
                continue;
            }
            bool ok;
            T* row = dst_row(ktl, g + j * hg, ok);
            if (ok) {
                *reinterpret_cast<uint4*>(row + kc * N) = VecOps<T>::pack(ra);
                *reinterpret_cast<uint4*>(row + half + kc * N) = VecOps<T>::pack(rb);
            }
        }
    }
    if (INSERT && bulk_st) {
        // every destination row is one contiguous run of H*D elements: one
        // shared->global bulk copy per K and V row, issued by one thread,
        // which waits until they have read shared memory before the CTA exits
        ptx::fence_proxy_async_smem();
        __syncthreads();
        if (threadIdx.x == 0) {
            const uint32_t rb = (uint32_t)(rowe * sizeof(T));
            for (int tl = 0; tl < nt; ++tl) {
                bool ok;
                T* row = dst_row(tl, 0, ok);
                if (!ok) continue;
                ptx::bulk_s2g(row, ksm + tl * rowe, rb);
                ptx::bulk_s2g(row + dkv, vsm + tl * rowe, rb);
            }
            ptx::bulk_commit();
            ptx::bulk_wait_read<0>();
        }
        return;
    }
    if (INSERT) {
#pragma unroll
        for (int j = 0; j < 2 * HPT; ++j) {
            const int vi = threadIdx.x + j * blockDim.x;
            if (vi < vitems) {
                const int c = vi % (2 * hc), r = vi / (2 * hc);
                const int h = r % num_heads, tl = r / num_heads;
                bool ok;
                T* row = dst_row(tl, h, ok);
                if (ok) stg_stream(row + dkv + c * N, *reinterpret_cast<const uint4*>(vsm + tl * rowe + h * 2 * half + c * N));
            }
        }
    }
}

// Tokens per CTA for rope_tokens_kernel with `hpt` heads per thread: one K
// item per thread (2*hpt V vectors per thread for the insert); 0 when the
// shape does not fit.
int tokens_per_block(int H, int half, int N, int hpt, int elem_bytes, bool insert) {
    if (half % N || H % hpt) return 0;
    const int per_token = (H / hpt) * (half / N);
    if (per_token > 256) return 0;
    int tpb = 256 / per_token;
    // angle table + staged K (and V) rows within the default 48 KB of shared memory
    const int per_tok_smem = (half / 2) * 16 + H * 2 * half * elem_bytes * (insert ? 2 : 1) + (insert ? 8 : 0);
    return std::min(tpb, (48 * 1024 - half * 4) / per_tok_smem);
}
size_t rope_tokens_smem(int tpb, int H, int half, int elem_bytes, bool insert) {
    return (size_t)tpb * ((half / 2) * 16 + (size_t)H * 2 * half * elem_bytes * (insert ? 2 : 1) + (insert ? 8 : 0)) +
           (size_t)half * 4;
}

template <typename T>
int launch_rope(void* k, int T_, int H, int D, int64_t ts, int64_t hs, const int32_t* orig,
                const int32_t* tgt, float theta, cudaStream_t st) {
    const int half = D / 2;
    FreqTable ft = make_freqs(theta, half);
    constexpr int N = VecOps<T>::N;
    bool vec = (half % N == 0) && ((reinterpret_cast<uintptr_t>(k) & 15) == 0) &&
               ((ts * (int64_t)sizeof(T)) % 16 == 0) && ((hs * (int64_t)sizeof(T)) % 16 == 0);
    int threads = 0, cpr = 0, kt = 0;
    const int tt = 16;
    // The row-parallel kernel measured slower than rope_remap_kernel for the
    // in-place case (56.5 vs 34.5 us at config 2); kept for the insert path.
    const int hpt = (H % 2 == 0) ? 2 : 1;        // heads per thread sharing one table read
    const int tpb_t = vec ? tokens_per_block(H, half, N, hpt, (int)sizeof(T), false) : 0;
    if (tpb_t > 0) {
        size_t smem = rope_tokens_smem(tpb_t, H, half, (int)sizeof(T), false);
        auto kern = hpt == 2 ? rope_tokens_kernel<T, false, 2> : rope_tokens_kernel<T, false, 1>;
        const int64_t es = sizeof(T);
        LaunchOrderGuard order;              // held until the launch below is issued
        const ByteRange krows = byte_span(k, ((int64_t)(T_ - 1) * ts + (int64_t)(H - 1) * hs + D) * es);
        const ByteRange reads[3] = {krows, byte_span(orig, (int64_t)T_ * 4), byte_span(tgt, tgt ? (int64_t)T_ * 4 : 0)};
        const int early = claim_early_reads(st, reads, 3, &krows, 1) && ts >= 0 && hs >= 0 ? 1 : 0;
        if (launch_pdl(kern, dim3((T_ + tpb_t - 1) / tpb_t), dim3(256), smem, st, (T*)k, (const T*)k,
                       (const T*)nullptr, T_, H, half, ts, hs, ts, hs, (int64_t)0, (int64_t)0, 1,
                       (const int32_t*)nullptr, 0, (int8_t*)nullptr, (int32_t*)nullptr, 0, orig, tgt, ft, tpb_t,
                       (int*)nullptr, 0, early) != cudaSuccess)
            return check_launch("rope_remap");
    } else if (vec && rows_shape<T>(H, D, tt, threads, cpr, kt)) {
        size_t smem = (size_t)2 * tt * half * sizeof(float);
        launch_rows<T, 0>(kt, dim3((T_ + tt - 1) / tt), threads, smem, st, (T*)k, (const T*)k, nullptr, T_, H, half,
                          cpr, ts, hs, ts, hs, 0, 0, 0, nullptr, 0, nullptr, nullptr, 0, orig, tgt, ft, tt, nullptr);
    } else if (vec) {
        int per_token = H * (half / N);
        int tpb = per_token >= 256 ? 1 : (256 / per_token);
        if (tpb > 64) tpb = 64;
        int grid = (T_ + tpb - 1) / tpb;
        size_t smem = (size_t)2 * tpb * half * sizeof(float);
        rope_remap_kernel<T><<<grid, 256, smem, st>>>((T*)k, T_, H, half, ts, hs, orig, tgt, ft, tpb);
    } else {
        int64_t total = (int64_t)T_ * H * half;
        int grid = (int)((total + 255) / 256);
        rope_remap_scalar_kernel<T><<<grid, 256, 0, st>>>((T*)k, T_, H, half, ts, hs, orig, tgt, ft);
    }
    return check_launch("rope_remap");
}

// ------------------------------------------------------------------ evict
// kessie_kernels_v2.hip:393-407 -- identical rule, used by the legacy launcher.
__global__ void page_evict_legacy_kernel(int8_t* __restrict__ valid, const int32_t* __restrict__ pos,
                                         int32_t* __restrict__ count, int thr, int P) {
    int p = blockIdx.x * blockDim.x + threadIdx.x;
    bool hit = false;
    if (p < P && valid[p] == 1 && pos[p] < thr) { valid[p] = 0; hit = true; }
    unsigned m = __ballot_sync(0xffffffffu, hit);
    if ((threadIdx.x & 31) == 0 && m) atomicAdd(count, __popc(m));
}

constexpr int kTile = 4096;          // pages per compaction tile
constexpr int kTileThreads = 1024;   // 4 pages per thread

size_t evict_ws(int P) {
    int tiles = (P + kTile - 1) / kTile;
    return align_up((size_t)P, 256) + align_up((size_t)tiles * 4, 256);
}

// Pass 1 of the ordered compaction: per page decide the flag, update state,
// write the flag byte and the tile's count.
// mode 0: eviction (valid/allocated update); mode 1: list pages with valid != 0.
__global__ void __launch_bounds__(kTileThreads) compact_flags_kernel(
    int8_t* __restrict__ valid, const int32_t* __restrict__ pos, int8_t* __restrict__ alloc, int P,
    int thr, int mode, uint8_t* __restrict__ flags, int32_t* __restrict__ tile_counts) {
    __shared__ int warp_sums[kTileThreads / 32];
    const int base = blockIdx.x * kTile + threadIdx.x * 4;
    int cnt = 0;
    uint32_t fl = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        int p = base + i;
        if (p >= P) break;
        int v = valid[p];
        bool f;
        if (mode == 1) {
            f = v != 0;
        } else {
            bool hit = (v == 1) && (pos[p] < thr);
            if (hit) { valid[p] = 0; v = 0; }
            if (alloc) {
                f = (alloc[p] == 1) && (v == 0);
                if (f) alloc[p] = 0;
            } else {
                f = hit;
            }
        }
        fl |= (uint32_t)f << (8 * i);
        cnt += f;
    }
    if (base + 3 < P) {
        *reinterpret_cast<uint32_t*>(flags + base) = fl;
    } else {
        for (int i = 0; i < 4 && base + i < P; ++i) flags[base + i] = (fl >> (8 * i)) & 1;
    }
    int w = __reduce_add_sync(0xffffffffu, cnt);
    if ((threadIdx.x & 31) == 0) warp_sums[threadIdx.x >> 5] = w;
    __syncthreads();
    if (threadIdx.x < 32) {
        int s = __reduce_add_sync(0xffffffffu, warp_sums[threadIdx.x]);
        if (threadIdx.x == 0) tile_counts[blockIdx.x] = s;
    }
}

// Pass 2: exclusive prefix over earlier tiles + in-tile scan, write ids in
// ascending page order.  Block 0 also writes the total.
__global__ void __launch_bounds__(kTileThreads) compact_scatter_kernel(
    const uint8_t* __restrict__ flags, const int32_t* __restrict__ tile_counts, int P, int tiles,
    int32_t* __restrict__ out_count, int32_t* __restrict__ out_ids) {
    __shared__ int warp_sums[kTileThreads / 32];
    __shared__ int s_prefix, s_total;
    // prefix of earlier tiles (and total) -- tiles is small (P/4096)
    int pre = 0, tot = 0;
    for (int i = threadIdx.x; i < tiles; i += blockDim.x) {
        int c = tile_counts[i];
        tot += c;
        if (i < (int)blockIdx.x) pre += c;
    }
    pre = __reduce_add_sync(0xffffffffu, pre);
    tot = __reduce_add_sync(0xffffffffu, tot);
    if ((threadIdx.x & 31) == 0) warp_sums[threadIdx.x >> 5] = pre;
    __syncthreads();
    if (threadIdx.x < 32) {
        int s = __reduce_add_sync(0xffffffffu, warp_sums[threadIdx.x]);
        if (threadIdx.x == 0) s_prefix = s;
    }
    __syncthreads();
    if ((threadIdx.x & 31) == 0) warp_sums[threadIdx.x >> 5] = tot;
    __syncthreads();
    if (threadIdx.x < 32) {
        int s = __reduce_add_sync(0xffffffffu, warp_sums[threadIdx.x]);
        if (threadIdx.x == 0) s_total = s;
    }
    __syncthreads();
    if (blockIdx.x == 0 && threadIdx.x == 0 && out_count) *out_count = s_total;
    if (!out_ids) return;

    const int base = blockIdx.x * kTile + threadIdx.x * 4;
    uint32_t fl = 0;
    for (int i = 0; i < 4; ++i)
        if (base + i < P) fl |= (uint32_t)(flags[base + i] & 1) << (8 * i);
    int cnt = __popc(fl);
    // warp inclusive scan
    int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    __syncthreads();
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int v = warp_sums[lane];
        int s = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        warp_sums[lane] = s - v;   // exclusive
    }
    __syncthreads();
    int off = s_prefix + warp_sums[warp] + incl - cnt;
    for (int i = 0; i < 4; ++i)
        if ((fl >> (8 * i)) & 1) out_ids[off++] = base + i;
}

int run_compaction(int8_t* valid, const int32_t* pos, int8_t* alloc, int P, int thr, int mode,
                   int32_t* count, int32_t* ids, void* ws, size_t wsb, cudaStream_t st) {
    if (P < 0) return set_error(KESSIE_ERR_ARG, "num_pages < 0");
    if (P == 0) {
        if (count) cudaMemsetAsync(count, 0, 4, st);
        return check_launch("page compaction (empty)");
    }
    if (!valid || (mode == 0 && !pos)) return set_error(KESSIE_ERR_ARG, "null page_valid/page_positions");
    size_t need = evict_ws(P);
    if (!ws || wsb < need)
        return set_error(KESSIE_ERR_WORKSPACE, "workspace %zu bytes < required %zu", wsb, need);
    int tiles = (P + kTile - 1) / kTile;
    uint8_t* flags = static_cast<uint8_t*>(ws);
    int32_t* tc = reinterpret_cast<int32_t*>(static_cast<char*>(ws) + align_up((size_t)P, 256));
    compact_flags_kernel<<<tiles, kTileThreads, 0, st>>>(valid, pos, alloc, P, thr, mode, flags, tc);
    compact_scatter_kernel<<<tiles, kTileThreads, 0, st>>>(flags, tc, P, tiles, count, ids);
    return check_launch("page compaction");
}

// ------------------------------------------------------------------ insert / gather
struct PageGeom {
    int64_t page_stride, token_stride, kv_stride, head_stride;   // elements
    int max_pages, page_size, num_heads, head_dim;
};

// One CTA per destination page: items = (kv, head, 16B chunk); each item
// copies its vector for the page's tokens.  K vectors are rotated when
// orig != nullptr (cos/sin per token from smem).
template <typename T, bool REMAP>
__global__ void __launch_bounds__(256) page_insert_kernel(
    T* __restrict__ cache, PageGeom g, const T* __restrict__ nk, const T* __restrict__ nv,
    int64_t src_ts, int64_t src_hs, int num_tokens, const int32_t* __restrict__ page_ids,
    int8_t* __restrict__ valid, int32_t* __restrict__ positions, int conv_pos,
    const int32_t* __restrict__ orig, const int32_t* __restrict__ tgt, FreqTable ft, int* status) {
    extern __shared__ float sm[];
    const int pg = blockIdx.x;
    const int ps = g.page_size;
    const int t0 = pg * ps;
    const int nt = min(ps, num_tokens - t0);
    const int phys = page_ids[pg];
    if (phys < 0 || phys >= g.max_pages) {       // kessie_kernels_v2.hip:441 skips silently
        if (threadIdx.x == 0) record_status(status, KESSIE_DEV_BAD_PAGE_ID);
        return;
    }
    constexpr int N = VecOps<T>::N;
    const int D = g.head_dim, half = D / 2;
    if (REMAP) {
        float* cs = sm;
        float* sn = sm + ps * half;
        for (int i = threadIdx.x; i < nt * half; i += blockDim.x) {
            int tl = i / half, d = i - tl * half;
            int t = t0 + tl;
            int target = tgt ? tgt[t] : conv_pos + t;
            float s, c;
            rope_sincos((float)(target - orig[t]) * ft.f[d], &s, &c);
            cs[i] = c; sn[i] = s;
        }
        __syncthreads();
    }
    if (threadIdx.x == 0 && valid) valid[phys] = 1;
    if (threadIdx.x == 0 && positions) positions[phys] = conv_pos + t0;
    T* page = cache + (int64_t)phys * g.page_stride;
    const int chunks = D / N;
    if (REMAP) {
        // K: items (head, low-half chunk) rotate pairs; V: items (head, chunk) copy.
        const int kitems = g.num_heads * (chunks / 2);
        const int vitems = g.num_heads * chunks;
        for (int i = threadIdx.x; i < kitems + vitems; i += blockDim.x) {
            if (i < kitems) {
                int h = i / (chunks / 2), c = i - h * (chunks / 2);
                const T* src = nk + (int64_t)t0 * src_ts + (int64_t)h * src_hs + c * N;
                T* dst = page + (int64_t)h * g.head_stride + c * N;
                for (int tl = 0; tl < nt; ++tl) {
                    uint4 lo = *reinterpret_cast<const uint4*>(src + (int64_t)tl * src_ts);
                    uint4 hi = *reinterpret_cast<const uint4*>(src + (int64_t)tl * src_ts + half);
                    rotate_pair<T>(lo, hi, sm + tl * half + c * N, sm + ps * half + tl * half + c * N);
                    *reinterpret_cast<uint4*>(dst + (int64_t)tl * g.token_stride) = lo;
                    *reinterpret_cast<uint4*>(dst + (int64_t)tl * g.token_stride + half) = hi;
                }
            } else {
                int j = i - kitems;
                int h = j / chunks, c = j - h * chunks;
                const T* src = nv + (int64_t)t0 * src_ts + (int64_t)h * src_hs + c * N;
                T* dst = page + g.kv_stride + (int64_t)h * g.head_stride + c * N;
#pragma unroll 4
                for (int tl = 0; tl < nt; ++tl)
                    *reinterpret_cast<uint4*>(dst + (int64_t)tl * g.token_stride) =
                        ldg_stream(src + (int64_t)tl * src_ts);
            }
        }
    } else {
        const int items = 2 * g.num_heads * chunks;
        for (int i = threadIdx.x; i < items; i += blockDim.x) {
            int kv = i / (g.num_heads * chunks);
            int r = i - kv * g.num_heads * chunks;
            int h = r / chunks, c = r - h * chunks;
            const T* src = (kv ? nv : nk) + (int64_t)t0 * src_ts + (int64_t)h * src_hs + c * N;
            T* dst = page + kv * g.kv_stride + (int64_t)h * g.head_stride + c * N;
#pragma unroll 4
            for (int tl = 0; tl < nt; ++tl)
                *reinterpret_cast<uint4*>(dst + (int64_t)tl * g.token_stride) =
                    ldg_stream(src + (int64_t)tl * src_ts);
        }
    }
}

// Legacy element-wise insert (kessie_kernels_v2.hip:414-456) for shapes the
// vector path cannot take (head_dim not a multiple of 8, unaligned rows).
template <typename T>
__global__ void page_insert_scalar_kernel(T* __restrict__ cache, PageGeom g, const T* __restrict__ nk,
                                          const T* __restrict__ nv, int64_t src_ts, int64_t src_hs,
                                          int num_tokens, const int32_t* __restrict__ page_ids,
                                          int8_t* __restrict__ valid, int32_t* __restrict__ positions,
                                          int conv_pos, int* status) {
    int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int64_t total = (int64_t)num_tokens * g.num_heads * g.head_dim;
    if (gid >= total) return;
    int d = (int)(gid % g.head_dim);
    int64_t r = gid / g.head_dim;
    int h = (int)(r % g.num_heads);
    int t = (int)(r / g.num_heads);
    int pg = t / g.page_size, in_pg = t % g.page_size;
    int phys = page_ids[pg];
    if (phys < 0 || phys >= g.max_pages) {
        if (in_pg == 0 && h == 0 && d == 0) record_status(status, KESSIE_DEV_BAD_PAGE_ID);
        return;
    }
    int64_t base = (int64_t)phys * g.page_stride + (int64_t)in_pg * g.token_stride + (int64_t)h * g.head_stride + d;
    int64_t src = (int64_t)t * src_ts + (int64_t)h * src_hs + d;
    cache[base] = nk[src];
    cache[base + g.kv_stride] = nv[src];
    if (in_pg == 0 && h == 0 && d == 0) {
        if (valid) valid[phys] = 1;
        if (positions) positions[phys] = conv_pos + t;
    }
}

// One CTA per gathered page: items (kv, head, chunk) copy their vector for
// all page_size tokens into the dense [n*ps, H, D] outputs.
template <typename T>
__global__ void __launch_bounds__(256) page_gather_kernel(const T* __restrict__ cache, PageGeom g,
                                                           const int32_t* __restrict__ ids,
                                                           T* __restrict__ ok, T* __restrict__ ov,
                                                           int* status) {
    const int i = blockIdx.x;
    const int phys = ids[i];
    const bool bad = phys < 0 || phys >= g.max_pages;
    if (bad && threadIdx.x == 0) record_status(status, KESSIE_DEV_BAD_PAGE_ID);
    constexpr int N = VecOps<T>::N;
    const int chunks = g.head_dim / N;
    const int H = g.num_heads, ps = g.page_size;
    const int64_t orow = (int64_t)H * g.head_dim;            // dense token stride
    const int items = 2 * H * chunks;
    const T* page = cache + (bad ? 0 : (int64_t)phys * g.page_stride);
    for (int it = threadIdx.x; it < items; it += blockDim.x) {
        int kv = it / (H * chunks);
        int r = it - kv * H * chunks;
        int h = r / chunks, c = r - h * chunks;
        T* out = kv ? ov : ok;
        if (!out) continue;
        const T* src = page + kv * g.kv_stride + (int64_t)h * g.head_stride + c * N;
        T* dst = out + (int64_t)i * ps * orow + (int64_t)h * g.head_dim + c * N;
        if (bad) {
            for (int t = 0; t < ps; ++t) *reinterpret_cast<uint4*>(dst + t * orow) = make_uint4(0, 0, 0, 0);
            continue;
        }
        if (ps == 16) {
            uint4 v[16];
#pragma unroll
            for (int t = 0; t < 16; ++t) v[t] = ldg_stream(src + (int64_t)t * g.token_stride);
#pragma unroll
            for (int t = 0; t < 16; ++t) stg_stream(dst + t * orow, v[t]);
        } else {
#pragma unroll 4
            for (int t = 0; t < ps; ++t) stg_stream(dst + t * orow, ldg_stream(src + (int64_t)t * g.token_stride));
        }
    }
}

template <typename T>
__global__ void page_gather_scalar_kernel(const T* __restrict__ cache, PageGeom g, const int32_t* __restrict__ ids,
                                          int n, T* __restrict__ ok, T* __restrict__ ov, int* status) {
    int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int64_t total = (int64_t)n * g.page_size * g.num_heads * g.head_dim;
    if (gid >= total) return;
    int d = (int)(gid % g.head_dim);
    int64_t r = gid / g.head_dim;
    int h = (int)(r % g.num_heads);
    int64_t tok = r / g.num_heads;
    int i = (int)(tok / g.page_size), s = (int)(tok % g.page_size);
    int phys = ids[i];
    bool bad = phys < 0 || phys >= g.max_pages;
    if (bad && s == 0 && h == 0 && d == 0) record_status(status, KESSIE_DEV_BAD_PAGE_ID);
    int64_t src = (int64_t)phys * g.page_stride + (int64_t)s * g.token_stride + (int64_t)h * g.head_stride + d;
    if (ok) ok[gid] = bad ? from_f32<T>(0.f) : cache[src];
    if (ov) ov[gid] = bad ? from_f32<T>(0.f) : cache[src + g.kv_stride];
}

// kessie_hip_kernels.py:408-412: w = 1, then (j / max(cs-1,1))^alpha for j < cs.
__global__ void fog_weights_kernel(float* __restrict__ w, int n, int cs, float alpha) {
    int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= n) return;
    float v = 1.f;
    if (alpha > 0.f && cs > 0 && j < cs) v = powf(__fdiv_rn((float)j, (float)max(cs - 1, 1)), alpha);
    w[j] = v;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }


template <typename T>
int launch_insert(void* cache, const PageGeom& g, const void* nk, const void* nv, int64_t sts, int64_t shs,
                  int T_, const int32_t* ids, int8_t* valid, int32_t* positions, int conv_pos,
                  const int32_t* orig, const int32_t* tgt, float theta, cudaStream_t st) {
    constexpr int N = VecOps<T>::N;
    const int es = sizeof(T);
    bool vec = g.head_dim % (2 * N) == 0 && aligned16(cache) && aligned16(nk) && aligned16(nv) &&
               (g.page_stride * es) % 16 == 0 && (g.token_stride * es) % 16 == 0 &&
               (g.kv_stride * es) % 16 == 0 && (g.head_stride * es) % 16 == 0 &&
               (sts * es) % 16 == 0 && (shs * es) % 16 == 0;
    int* status = device_status_ptr();
    int pages = (T_ + g.page_size - 1) / g.page_size;
    if (pages == 0) return check_launch("page_insert (empty)");
    int threads = 0, cpr = 0, kt = 0;
    const int hpt = (g.num_heads % 2 == 0) ? 2 : 1;
    const int tpb_i = (orig && vec) ? tokens_per_block(g.num_heads, g.head_dim / 2, N, hpt, es, true) : 0;
    if (tpb_i > 0) {
        FreqTable ft = make_freqs(theta, g.head_dim / 2);
        size_t smem = rope_tokens_smem(tpb_i, g.num_heads, g.head_dim / 2, es, true);
        auto kern = hpt == 2 ? rope_tokens_kernel<T, true, 2> : rope_tokens_kernel<T, true, 1>;
        // destination rows of all heads contiguous: K and V rows leave as bulk copies
        const int bulk_st = (g.head_stride == g.head_dim && ((int64_t)g.num_heads * g.head_dim * es) % 16 == 0) ? 1 : 0;
        LaunchOrderGuard order;              // held until the launch below is issued
        const int64_t rows_e = (int64_t)(T_ - 1) * sts + (int64_t)(g.num_heads - 1) * shs + g.head_dim;
        const ByteRange reads[5] = {byte_span(nk, rows_e * es), byte_span(nv, rows_e * es),
                                    byte_span(ids, (int64_t)pages * 4), byte_span(orig, (int64_t)T_ * 4),
                                    byte_span(tgt, tgt ? (int64_t)T_ * 4 : 0)};
        const int64_t cache_e = (int64_t)(g.max_pages - 1) * g.page_stride + (int64_t)(g.page_size - 1) * g.token_stride +
                                g.kv_stride + (int64_t)(g.num_heads - 1) * g.head_stride + g.head_dim;
        const ByteRange writes[3] = {byte_span(cache, cache_e * es), byte_span(valid, valid ? g.max_pages : 0),
                                     byte_span(positions, positions ? (int64_t)g.max_pages * 4 : 0)};
        const bool fwd = sts >= 0 && shs >= 0 && g.page_stride >= 0 && g.token_stride >= 0 && g.kv_stride >= 0 &&
                         g.head_stride >= 0;
        const int early = claim_early_reads(st, reads, 5, writes, 3) && fwd ? 1 : 0;
        if (launch_pdl(kern, dim3((T_ + tpb_i - 1) / tpb_i), dim3(256), smem, st, (T*)cache, (const T*)nk,
                       (const T*)nv, T_, g.num_heads, g.head_dim / 2, sts, shs, g.token_stride, g.head_stride,
                       g.kv_stride, g.page_stride, g.page_size, ids, g.max_pages, valid, positions, conv_pos, orig,
                       tgt, ft, tpb_i, status, bulk_st, early) != cudaSuccess)
            return check_launch("page_insert");
    } else if (orig && vec && g.page_size <= 256 && rows_shape<T>(g.num_heads, g.head_dim, g.page_size, threads, cpr, kt)) {
        FreqTable ft = make_freqs(theta, g.head_dim / 2);
        size_t smem = (size_t)2 * g.page_size * (g.head_dim / 2) * sizeof(float);
        if (smem > 48 * 1024) {
            cudaFuncSetAttribute(rope_rows_kernel<T, 1, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            cudaFuncSetAttribute(rope_rows_kernel<T, 1, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            cudaFuncSetAttribute(rope_rows_kernel<T, 1, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            cudaFuncSetAttribute(rope_rows_kernel<T, 1, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            cudaFuncSetAttribute(rope_rows_kernel<T, 1, 16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        }
        launch_rows<T, 1>(kt, dim3(pages), threads, smem, st, (T*)cache, (const T*)nk, (const T*)nv, T_, g.num_heads,
                          g.head_dim / 2, cpr, sts, shs, g.token_stride, g.head_stride, g.kv_stride, g.page_stride,
                          g.page_size, ids, g.max_pages, valid, positions, conv_pos, orig, tgt, ft, g.page_size, status);
    } else if (orig) {
        if (!vec) return set_error(KESSIE_ERR_UNSUPPORTED, "fused insert+remap needs 16-byte aligned rows and head_dim %% %d == 0", 2 * N);
        if (g.head_dim / 2 > kMaxHalf) return set_error(KESSIE_ERR_UNSUPPORTED, "head_dim > %d", 2 * kMaxHalf);
        FreqTable ft = make_freqs(theta, g.head_dim / 2);
        size_t smem = (size_t)2 * g.page_size * (g.head_dim / 2) * sizeof(float);
        if (smem > 200 * 1024) return set_error(KESSIE_ERR_UNSUPPORTED, "page_size too large for fused remap");
        if (smem > 48 * 1024)
            cudaFuncSetAttribute(page_insert_kernel<T, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        page_insert_kernel<T, true><<<pages, 256, smem, st>>>((T*)cache, g, (const T*)nk, (const T*)nv, sts, shs, T_,
                                                               ids, valid, positions, conv_pos, orig, tgt, ft, status);
    } else if (vec) {
        FreqTable ft{};
        page_insert_kernel<T, false><<<pages, 256, 0, st>>>((T*)cache, g, (const T*)nk, (const T*)nv, sts, shs, T_,
                                                             ids, valid, positions, conv_pos, nullptr, nullptr, ft, status);
    } else {
        int64_t total = (int64_t)T_ * g.num_heads * g.head_dim;
        page_insert_scalar_kernel<T><<<(unsigned)((total + 255) / 256), 256, 0, st>>>(
            (T*)cache, g, (const T*)nk, (const T*)nv, sts, shs, T_, ids, valid, positions, conv_pos, status);
    }
    return check_launch("page_insert");
}

template <typename T>
int launch_gather(const void* cache, const PageGeom& g, const int32_t* ids, int n, void* ok, void* ov, cudaStream_t st) {
    constexpr int N = VecOps<T>::N;
    const int es = sizeof(T);
    int* status = device_status_ptr();
    if (n == 0) return check_launch("page_gather (empty)");
    bool vec = g.head_dim % N == 0 && aligned16(cache) && (!ok || aligned16(ok)) && (!ov || aligned16(ov)) &&
               (g.page_stride * es) % 16 == 0 && (g.token_stride * es) % 16 == 0 &&
               (g.kv_stride * es) % 16 == 0 && (g.head_stride * es) % 16 == 0;
    const int64_t R = (int64_t)g.num_heads * g.head_dim * es;
    if (vec && g.head_stride == g.head_dim && bulk_ok(R)) {
        BulkArgs a{};
        a.cache = static_cast<const char*>(cache);
        a.page_b = g.page_stride * es; a.token_b = g.token_stride * es; a.kv_b = g.kv_stride * es;
        a.max_pages = g.max_pages; a.ps = g.page_size; a.ids = ids;
        a.rk = (char*)ok; a.rv = (char*)ov; a.R = (int)R; a.units = n; a.status = status;
        if (launch_gather_bulk(a, st)) return check_launch("page_gather (bulk)");
    }
    if (vec) {
        page_gather_kernel<T><<<n, 256, 0, st>>>((const T*)cache, g, ids, (T*)ok, (T*)ov, status);
    } else {
        int64_t total = (int64_t)n * g.page_size * g.num_heads * g.head_dim;
        page_gather_scalar_kernel<T><<<(unsigned)((total + 255) / 256), 256, 0, st>>>((const T*)cache, g, ids, n, (T*)ok, (T*)ov, status);
    }
    return check_launch("page_gather");
}

}  // namespace
}  // namespace kessie

using namespace kessie;

// ============================================================== C ABI
extern "C" {

void launch_kessie_rope_remap(void* k_data, const void* orig_positions, const void* target_positions,
                              float rope_theta, int num_tokens, int num_heads, int half_dim, void* stream) {
    if (!k_data || !orig_positions || !target_positions || num_tokens < 0 || num_heads <= 0 ||
        half_dim <= 0 || half_dim > kMaxHalf) {
        set_error(KESSIE_ERR_ARG, "launch_kessie_rope_remap: bad arguments (half_dim=%d)", half_dim);
        return;
    }
    if (num_tokens == 0) { clear_error(); return; }
    int64_t D = 2 * (int64_t)half_dim;
    launch_rope<__half>(k_data, num_tokens, num_heads, (int)D, (int64_t)num_heads * D, D,
                        (const int32_t*)orig_positions, (const int32_t*)target_positions, rope_theta,
                        as_stream(stream));
}

int kessie_rope_remap_v2(void* k_data, int dtype, int num_tokens, int num_heads, int head_dim,
                         int64_t token_stride, int64_t head_stride, const int32_t* orig_positions,
                         const int32_t* target_positions, float rope_theta, void* stream) {
    NvtxRange nvtx_range("kessie_rope_remap_v2");
    if (!dtype_ok(dtype)) return set_error(KESSIE_ERR_UNSUPPORTED, "rope_remap_v2: dtype %d", dtype);
    if (num_tokens < 0 || num_heads <= 0 || head_dim <= 0 || (head_dim & 1) || head_dim / 2 > kMaxHalf)
        return set_error(KESSIE_ERR_ARG, "rope_remap_v2: bad shape T=%d H=%d D=%d", num_tokens, num_heads, head_dim);
    if (num_tokens == 0) { clear_error(); return 0; }
    if (!k_data || !orig_positions || !target_positions) return set_error(KESSIE_ERR_ARG, "rope_remap_v2: null pointer");
    if (token_stride < head_dim || head_stride < head_dim)
        return set_error(KESSIE_ERR_ARG, "rope_remap_v2: strides smaller than head_dim");
    cudaStream_t st = as_stream(stream);
    switch (dtype) {
        case KESSIE_DTYPE_F16: return launch_rope<__half>(k_data, num_tokens, num_heads, head_dim, token_stride, head_stride, orig_positions, target_positions, rope_theta, st);
        case KESSIE_DTYPE_BF16: return launch_rope<__nv_bfloat16>(k_data, num_tokens, num_heads, head_dim, token_stride, head_stride, orig_positions, target_positions, rope_theta, st);
        default: return launch_rope<float>(k_data, num_tokens, num_heads, head_dim, token_stride, head_stride, orig_positions, target_positions, rope_theta, st);
    }
}

void launch_kessie_page_evict(void* page_valid, const void* page_positions, void* evict_count,
                              int evict_before_pos, int num_pages, void* stream) {
    if (num_pages <= 0) { clear_error(); return; }
    if (!page_valid || !page_positions || !evict_count) {
        set_error(KESSIE_ERR_ARG, "launch_kessie_page_evict: null pointer");
        return;
    }
    page_evict_legacy_kernel<<<(num_pages + 255) / 256, 256, 0, as_stream(stream)>>>(
        (int8_t*)page_valid, (const int32_t*)page_positions, (int32_t*)evict_count, evict_before_pos, num_pages);
    check_launch("page_evict");
}

size_t kessie_page_evict_workspace_size(int num_pages) { return num_pages > 0 ? evict_ws(num_pages) : 0; }

int kessie_page_evict_v2(int8_t* page_valid, const int32_t* page_positions, int8_t* page_allocated,
                         int num_pages, int evict_before_pos, int32_t* freed_count, int32_t* freed_ids,
                         void* workspace, size_t workspace_bytes, void* stream) {
    NvtxRange nvtx_range("kessie_page_evict_v2");
    return run_compaction(page_valid, page_positions, page_allocated, num_pages, evict_before_pos, 0,
                          freed_count, freed_ids, workspace, workspace_bytes, as_stream(stream));
}

int kessie_page_list_valid_v2(const int8_t* page_valid, int num_pages, int32_t* count, int32_t* ids,
                              void* workspace, size_t workspace_bytes, void* stream) {
    NvtxRange nvtx_range("kessie_page_list_valid_v2");
    return run_compaction(const_cast<int8_t*>(page_valid), nullptr, nullptr, num_pages, 0, 1, count, ids,
                          workspace, workspace_bytes, as_stream(stream));
}

void launch_kessie_page_insert(void* kv_cache, const void* new_keys, const void* new_values,
                               const void* target_page_ids, void* page_valid, void* page_positions,
                               int conv_pos, int num_tokens, int num_heads, int head_dim, int page_size,
                               int max_pages, void* stream) {
    if (num_tokens <= 0) { clear_error(); return; }
    if (!kv_cache || !new_keys || !new_values || !target_page_ids || num_heads <= 0 || head_dim <= 0 ||
        page_size <= 0 || max_pages <= 0) {
        set_error(KESSIE_ERR_ARG, "launch_kessie_page_insert: bad arguments");
        return;
    }
    PageGeom g;
    g.head_stride = head_dim;
    g.kv_stride = (int64_t)num_heads * head_dim;
    g.token_stride = 2 * g.kv_stride;
    g.page_stride = (int64_t)page_size * g.token_stride;
    g.max_pages = max_pages; g.page_size = page_size; g.num_heads = num_heads; g.head_dim = head_dim;
    launch_insert<__half>(kv_cache, g, new_keys, new_values, (int64_t)num_heads * head_dim, head_dim, num_tokens,
                          (const int32_t*)target_page_ids, (int8_t*)page_valid, (int32_t*)page_positions,
                          conv_pos, nullptr, nullptr, 0.f, as_stream(stream));
}

int kessie_page_insert_v2(void* kv_cache, int dtype, int64_t page_stride, int64_t token_stride, int64_t kv_stride,
                          int64_t head_stride, int max_pages, int page_size, const void* new_keys,
                          const void* new_values, int64_t src_token_stride, int64_t src_head_stride, int num_tokens,
                          int num_heads, int head_dim, const int32_t* target_page_ids, int8_t* page_valid,
                          int32_t* page_positions, int conv_pos, const int32_t* orig_positions,
                          const int32_t* target_positions, float rope_theta, void* stream) {
    NvtxRange nvtx_range("kessie_page_insert_v2");
    if (!dtype_ok(dtype)) return set_error(KESSIE_ERR_UNSUPPORTED, "page_insert_v2: dtype %d", dtype);
    if (num_tokens < 0 || num_heads <= 0 || head_dim <= 0 || page_size <= 0 || max_pages <= 0)
        return set_error(KESSIE_ERR_ARG, "page_insert_v2: bad shape");
    if (num_tokens == 0) { clear_error(); return 0; }
    if (!kv_cache || !new_keys || !new_values || !target_page_ids)
        return set_error(KESSIE_ERR_ARG, "page_insert_v2: null pointer");
    if (orig_positions && (head_dim & 1)) return set_error(KESSIE_ERR_ARG, "page_insert_v2: odd head_dim with remap");
    PageGeom g{page_stride, token_stride, kv_stride, head_stride, max_pages, page_size, num_heads, head_dim};
    cudaStream_t st = as_stream(stream);
    switch (dtype) {
        case KESSIE_DTYPE_F16: return launch_insert<__half>(kv_cache, g, new_keys, new_values, src_token_stride, src_head_stride, num_tokens, target_page_ids, page_valid, page_positions, conv_pos, orig_positions, target_positions, rope_theta, st);
        case KESSIE_DTYPE_BF16: return launch_insert<__nv_bfloat16>(kv_cache, g, new_keys, new_values, src_token_stride, src_head_stride, num_tokens, target_page_ids, page_valid, page_positions, conv_pos, orig_positions, target_positions, rope_theta, st);
        default: return launch_insert<float>(kv_cache, g, new_keys, new_values, src_token_stride, src_head_stride, num_tokens, target_page_ids, page_valid, page_positions, conv_pos, orig_positions, target_positions, rope_theta, st);
    }
}

int kessie_page_gather_v2(const void* kv_cache, int dtype, int64_t page_stride, int64_t token_stride,
                          int64_t kv_stride, int64_t head_stride, int max_pages, int page_size,
                          const int32_t* page_ids, int num_gather, int num_heads, int head_dim, void* out_keys,
                          void* out_values, void* stream) {
    NvtxRange nvtx_range("kessie_page_gather_v2");
    if (!dtype_ok(dtype)) return set_error(KESSIE_ERR_UNSUPPORTED, "page_gather_v2: dtype %d", dtype);
    if (num_gather < 0 || num_heads <= 0 || head_dim <= 0 || page_size <= 0 || max_pages <= 0)
        return set_error(KESSIE_ERR_ARG, "page_gather_v2: bad shape");
    if (num_gather == 0) { clear_error(); return 0; }
    if (!kv_cache || !page_ids || (!out_keys && !out_values)) return set_error(KESSIE_ERR_ARG, "page_gather_v2: null pointer");
    PageGeom g{page_stride, token_stride, kv_stride, head_stride, max_pages, page_size, num_heads, head_dim};
    cudaStream_t st = as_stream(stream);
    switch (dtype) {
        case KESSIE_DTYPE_F16: return launch_gather<__half>(kv_cache, g, page_ids, num_gather, out_keys, out_values, st);
        case KESSIE_DTYPE_BF16: return launch_gather<__nv_bfloat16>(kv_cache, g, page_ids, num_gather, out_keys, out_values, st);
        default: return launch_gather<float>(kv_cache, g, page_ids, num_gather, out_keys, out_values, st);
    }
}

int kessie_build_fog_weights_v2(float* out, int seq_len, int clear_start, float fog_alpha, void* stream) {
    NvtxRange nvtx_range("kessie_build_fog_weights_v2");
    if (seq_len < 0 || (seq_len > 0 && !out)) return set_error(KESSIE_ERR_ARG, "build_fog_weights_v2: bad arguments");
    if (seq_len == 0) { clear_error(); return 0; }
    fog_weights_kernel<<<(seq_len + 255) / 256, 256, 0, as_stream(stream)>>>(out, seq_len, clear_start, fog_alpha);
    return check_launch("build_fog_weights");
}

}  // extern "C"
