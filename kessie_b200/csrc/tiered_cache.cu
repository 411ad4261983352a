// tiered_cache.cu -- the HF tiered KV cache's device work (KeSSieCache,
// kessie_exp3.py:342-627) on per-layer stores that never move on append.
//
// Store layout per layer and K/V: [B, H, cap, D] elements, the live tokens at
// [lo, hi) of the cap axis.  key_cache / value_cache are views of the live
// range, so an append writes T tokens in place (the reference's torch.cat
// re-copies the whole cache every step) and an eviction moves lo.
//
// kessie_tiered_update_v2 (KeSSieCache.update, kessie_exp3.py:425-450): one
// launch appends the T new K and V tokens at hi and, with the fog on, writes
// the fogged V of the whole live range into a contiguous [B, H, S, D] buffer:
//   v_fog[s] = dtype(float(v[s]) * w(s)),  S = hi + T - lo,
//   w(s) = max((s / max(fc - 1, 1)) ^ alpha, 0.01) for s < fc, else 1,
//   fc = S - max(1, int(S * fog_start))       (_compute_fog_mask, :415-423)
// New tokens are read from the caller's tensors, never from the store written
// by the same launch.  Every row is moved in 16-byte vectors: one read and one
// write of the live V per step (HBM-bound), plus the T-token appends.
//
// kessie_strided_pack_v2 (evict_if_needed / recall_from_cpu, :452-533): one
// launch copies tokens [t0, t0 + n) of every (layer, K/V) store to or from a
// contiguous staging [M][B*H][n][D] (M = layers * 2), so an eviction is one
// pack + one device-to-host copy and a recall one host-to-device copy + one
// unpack.
#include "common.cuh"
#include "ptx.cuh"

#include <math.h>


namespace kessie {
namespace {

// w(s); the exponents torch's pow(tensor, scalar) evaluates without pow()
// (0.5, 1, 2, 3) take the same route, so the weights agree bit for bit there.
__device__ __forceinline__ float tiered_fog_weight(long long s, int fc, float den, float alpha, int alpha_mode) {
    if (s >= fc) return 1.f;
    const float x = (float)s / den;
    float w;
    switch (alpha_mode) {
        case 1: w = sqrtf(x); break;
        case 2: w = x; break;
        case 3: w = x * x; break;
        case 4: w = x * x * x; break;
        default: w = powf(x, alpha); break;
    }
    return fmaxf(w, 0.01f);
}

template <typename T>
__device__ __forceinline__ uint4 scale16(uint4 raw, float w) {
    constexpr int N = 16 / sizeof(T);
    union { uint4 u; T e[N]; } a;
    a.u = raw;
#pragma unroll
    for (int i = 0; i < N; ++i) a.e[i] = from_f32<T>(to_f32(a.e[i]) * w);
    return a.u;
}

struct TieredUpdateArgs {
    char* k_store;
    char* v_store;
    const char* k_new;
    const char* v_new;
    char* v_fog;                  // nullptr: fog off
    long long cap, lo, hi;        // tokens
    long long nsb, nsh, nst;      // new-token strides (bytes) for b, h, t
    int H, T, S, chunks;          // S = live tokens after the append; chunks = row bytes / 16
    int fc, alpha_mode;
    float den, alpha;
    int early;                    // issue the live-V loads before griddepcontrol.wait
};

constexpr int kItems = 4;                                  // 16-byte items in flight per thread (pack)
// The update keeps 8 in flight per thread: a layer's grid (392 CTAs at the
// decode-step shape, 3 per SM at 79 registers) then leaves SM slots for the
// next layer's CTAs to start their early reads while this one drains
// (4 items: 776 CTAs filled the 740 slots, 0.73 of HBM; 8: 0.78; 12 / 16
// drop to 2 CTAs per SM, 0.62 / 0.57).
constexpr int kUpdItems = 8;

// grid (x over the rows of one (b, h), y = b * H + h): rows [0, S) are the
// fogged V (or [0, T) the V append when the fog is off), then T K-append rows.
// Launched as a programmatic dependent of whatever precedes it on the stream
// (the previous layer's update in a decode step).  Every CTA waits for the
// preceding grid to complete (griddepcontrol.wait) and only then lets the next
// launch start (launch_dependents), so while a grid runs, every grid launched
// before its predecessor has completed.  With a.early the loads of the live V
// rows already in the store are issued BEFORE the wait, overlapping the
// preceding grid's drain: the host sets it only when the last programmatic
// launch of this library on this stream (claim_early_reads) wrote none of
// this V store, so the one grid that can still be running writes no byte
// these loads read.  Loads of the new
// tokens (written by the caller's producer) and every store follow the wait.
template <typename T, int CH>
__global__ void __launch_bounds__(256) tiered_update_kernel(TieredUpdateArgs a) {
    const int chunks = CH > 0 ? CH : a.chunks;
    const long long rb = (long long)chunks * 16;
    const int bh = blockIdx.y, b = bh / a.H, h = bh - b * a.H;
    const int s_old = (int)(a.hi - a.lo);
    const int vrows = a.v_fog ? a.S : a.T;
    const int items = (vrows + a.T) * chunks;
    char* vst = a.v_store + (long long)bh * a.cap * rb;
    char* kst = a.k_store + (long long)bh * a.cap * rb;
    const char* vnew = a.v_new + b * a.nsb + h * a.nsh;
    const char* knew = a.k_new + b * a.nsb + h * a.nsh;
    char* vfog = a.v_fog ? a.v_fog + (long long)bh * a.S * rb : nullptr;
    bool waited = !a.early;
    if (waited) {
        ptx::grid_dependency_wait();
        ptx::launch_dependents();
    }
    for (int base = blockIdx.x * 256 * kUpdItems + threadIdx.x; base < items; base += gridDim.x * 256 * kUpdItems) {
        uint4 raw[kUpdItems];
        const char* src[kUpdItems];
#pragma unroll
        for (int u = 0; u < kUpdItems; ++u) {
            const int i = base + u * 256;
            src[u] = nullptr;
            if (i >= items) break;
            const int r = i / chunks, c = i - r * chunks;
            const bool stored = vfog && r < vrows && r < s_old;
            if (r < vrows) {
                if (stored) src[u] = vst + (a.lo + r) * rb;
                else src[u] = vnew + (long long)(vfog ? r - s_old : r) * a.nst;
            } else {
                src[u] = knew + (long long)(r - vrows) * a.nst;
            }
            src[u] += c * 16;
            if (stored || waited) raw[u] = ldg_stream(src[u]);
        }
        if (!waited) {
            ptx::grid_dependency_wait();
            ptx::launch_dependents();
            waited = true;
#pragma unroll
            for (int u = 0; u < kUpdItems; ++u) {
                const int i = base + u * 256;
                if (i >= items) break;
                const int r = i / chunks;
                if (!(vfog && r < vrows && r < s_old)) raw[u] = ldg_stream(src[u]);
            }
        }
#pragma unroll
        for (int u = 0; u < kUpdItems; ++u) {
            const int i = base + u * 256;
            if (i >= items) break;
            const int r = i / chunks, c = i - r * chunks;
            if (r < vrows) {
                if (vfog) {
                    const float w = tiered_fog_weight(r, a.fc, a.den, a.alpha, a.alpha_mode);
                    stg_stream(vfog + r * rb + c * 16, scale16<T>(raw[u], w));
                    if (r >= s_old)
                        *reinterpret_cast<uint4*>(vst + (a.hi + r - s_old) * rb + c * 16) = raw[u];
                } else {
                    *reinterpret_cast<uint4*>(vst + (a.hi + r) * rb + c * 16) = raw[u];
                }
            } else {
                *reinterpret_cast<uint4*>(kst + (a.hi + r - vrows) * rb + c * 16) = raw[u];
            }
        }
    }
}

// Pack (unpack = 0) or unpack (1): grid (x over one store row's tokens,
// y = store * BH + row); row y of the staging is contiguous.
template <int CH>
__global__ void __launch_bounds__(256) strided_pack_kernel(const unsigned long long* __restrict__ bases,
                                                           const long long* __restrict__ pitches, int BH, int n,
                                                           int chunks_rt, char* __restrict__ staging, int unpack) {
    const int chunks = CH > 0 ? CH : chunks_rt;
    const long long rb = (long long)chunks * 16;
    const int m = blockIdx.y / BH, bh = blockIdx.y - m * BH;
    char* store = reinterpret_cast<char*>(bases[m]) + bh * pitches[m];
    char* stage = staging + (long long)blockIdx.y * n * rb;
    const int items = n * chunks;                          // one store row = n tokens x rb bytes, contiguous
    for (int base = blockIdx.x * 256 * kItems + threadIdx.x; base < items; base += gridDim.x * 256 * kItems) {
        uint4 v[kItems];
#pragma unroll
        for (int u = 0; u < kItems; ++u) {
            const int i = base + u * 256;
            if (i >= items) break;
            v[u] = ldg_stream((unpack ? stage : store) + (long long)i * 16);
        }
#pragma unroll
        for (int u = 0; u < kItems; ++u) {
            const int i = base + u * 256;
            if (i >= items) break;
            char* dst = (unpack ? store : stage) + (long long)i * 16;
            if (unpack) *reinterpret_cast<uint4*>(dst) = v[u];
            else stg_stream(dst, v[u]);
        }
    }
}

// x blocks for `items` per y row (`per_thread` 16-byte items per thread and
// batch): enough CTAs in total for the SMs, at most one item batch per thread
// when that fits.
int grid_x(long long items, long long rows_y, int per_thread) {
    const long long per = 256LL * per_thread;
    long long gx = (items + per - 1) / per;
    const long long cap = ((long long)sm_count() * 16 + rows_y - 1) / rows_y;
    if (gx > cap) gx = cap;
    return (int)(gx < 1 ? 1 : gx);
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace kessie

using namespace kessie;

extern "C" int kessie_tiered_update_v2(void* k_store, void* v_store, long long cap, long long lo, long long hi,
                                       const void* k_new, const void* v_new, long long new_stride_b,
                                       long long new_stride_h, long long new_stride_t, int B, int H, int T, int D,
                                       int dtype, void* v_fog, float fog_alpha, double fog_start, void* stream) {
    NvtxRange nvtx_range("kessie_tiered_update_v2");
    if (!k_store || !v_store || !k_new || !v_new || B <= 0 || H <= 0 || T < 0 || D <= 0 || !dtype_ok(dtype) ||
        lo < 0 || hi < lo || cap < hi + T)
        return set_error(KESSIE_ERR_ARG, "tiered_update_v2: bad arguments (0 <= lo <= hi, hi + T <= cap)");
    const int es = dtype_bytes(dtype);
    if (((long long)D * es) % 16)
        return set_error(KESSIE_ERR_ARG, "tiered_update_v2: head_dim * element size must be a multiple of 16");
    if (!al16(k_store) || !al16(v_store) || !al16(k_new) || !al16(v_new) || (v_fog && !al16(v_fog)) ||
        ((new_stride_b | new_stride_h | new_stride_t) * es) % 16)
        return set_error(KESSIE_ERR_ARG, "tiered_update_v2: 16-byte aligned buffers and strides required");
    const long long S = hi + T - lo;
    // fog active exactly when the reference's _compute_fog_mask returns a mask
    int fc = 0;
    if (fog_alpha > 0.f && S > 0) {
        long long cc = (long long)((double)S * fog_start);   // Python int(S * fog_start)
        if (cc < 1) cc = 1;
        fc = (int)(S - cc);
    }
    if (fc <= 0) v_fog = nullptr;
    if ((long long)B * H > 65535 || S > (1LL << 30) / (D * es / 16 + 1))
        return set_error(KESSIE_ERR_ARG, "tiered_update_v2: B * H <= 65535 and S * row chunks < 2^30");
    TieredUpdateArgs a;
    a.k_store = static_cast<char*>(k_store);
    a.v_store = static_cast<char*>(v_store);
    a.k_new = static_cast<const char*>(k_new);
    a.v_new = static_cast<const char*>(v_new);
    a.v_fog = static_cast<char*>(v_fog);
    a.cap = cap; a.lo = lo; a.hi = hi;
    a.nsb = new_stride_b * es; a.nsh = new_stride_h * es; a.nst = new_stride_t * es;
    a.H = H; a.T = T; a.S = (int)S; a.chunks = D * es / 16;
    a.fc = fc;
    a.den = (float)(fc - 1 > 1 ? fc - 1 : 1);
    a.alpha = fog_alpha;
    a.alpha_mode = fog_alpha == 0.5f ? 1 : fog_alpha == 1.f ? 2 : fog_alpha == 2.f ? 3 : fog_alpha == 3.f ? 4 : 0;
    const long long rows = (v_fog ? S : T) + T;
    if (rows == 0) { clear_error(); return 0; }
    cudaStream_t st = as_stream(stream);
    LaunchOrderGuard order;                  // held until the launch below is issued
    {
        const uintptr_t store_bytes = (uintptr_t)((long long)B * H * cap * a.chunks * 16);
        const uintptr_t kb = reinterpret_cast<uintptr_t>(k_store), vb = reinterpret_cast<uintptr_t>(v_store);
        const uintptr_t fb = reinterpret_cast<uintptr_t>(v_fog);
        const ByteRange w[3] = {{kb, kb + store_bytes}, {vb, vb + store_bytes},
                                v_fog ? ByteRange{fb, fb + (uintptr_t)((long long)B * H * S * a.chunks * 16)}
                                      : ByteRange{0, 0}};
        a.early = claim_early_reads(st, &w[1], 1, w, 3) && v_fog != nullptr ? 1 : 0;
    }
    const dim3 grid(grid_x(rows * a.chunks, (long long)B * H, kUpdItems), B * H);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t lerr = cudaSuccess;
    auto launch = [&](auto kern) { lerr = cudaLaunchKernelEx(&cfg, kern, a); };
    if (dtype == KESSIE_DTYPE_BF16) {
        if (a.chunks == 16) launch(tiered_update_kernel<__nv_bfloat16, 16>);
        else if (a.chunks == 8) launch(tiered_update_kernel<__nv_bfloat16, 8>);
        else launch(tiered_update_kernel<__nv_bfloat16, 0>);
    } else if (dtype == KESSIE_DTYPE_F16) {
        if (a.chunks == 16) launch(tiered_update_kernel<__half, 16>);
        else if (a.chunks == 8) launch(tiered_update_kernel<__half, 8>);
        else launch(tiered_update_kernel<__half, 0>);
    } else {
        if (a.chunks == 32) launch(tiered_update_kernel<float, 32>);
        else if (a.chunks == 16) launch(tiered_update_kernel<float, 16>);
        else launch(tiered_update_kernel<float, 0>);
    }
    if (lerr != cudaSuccess) {
        cudaGetLastError();
        return set_error(KESSIE_ERR_CUDA, "tiered_update: %s", cudaGetErrorString(lerr));
    }
    return check_launch("tiered_update");
}

extern "C" int kessie_strided_pack_v2(const unsigned long long* store_bases, const long long* store_pitch_bytes,
                                      int num_stores, int rows_per_store, long long tokens, int row_bytes,
                                      void* staging, int unpack, void* stream) {
    NvtxRange nvtx_range("kessie_strided_pack_v2");
    if (!store_bases || !store_pitch_bytes || !staging || num_stores <= 0 || rows_per_store <= 0 || tokens < 0 ||
        row_bytes <= 0 || row_bytes % 16 || !al16(staging))
        return set_error(KESSIE_ERR_ARG, "strided_pack_v2: bad arguments (row_bytes % 16 == 0, aligned staging)");
    if ((long long)num_stores * rows_per_store > 65535 || tokens * (row_bytes / 16) > (1LL << 30))
        return set_error(KESSIE_ERR_ARG, "strided_pack_v2: stores * rows <= 65535, tokens * row chunks < 2^30");
    if (tokens == 0) { clear_error(); return 0; }
    const int ch = row_bytes / 16, ys = num_stores * rows_per_store;
    const dim3 grid(grid_x(tokens * ch, ys, kItems), ys);
    cudaStream_t st = as_stream(stream);
    if (ch == 16)
        strided_pack_kernel<16><<<grid, 256, 0, st>>>(store_bases, store_pitch_bytes, rows_per_store, (int)tokens, ch,
                                                       static_cast<char*>(staging), unpack ? 1 : 0);
    else
        strided_pack_kernel<0><<<grid, 256, 0, st>>>(store_bases, store_pitch_bytes, rows_per_store, (int)tokens, ch,
                                                      static_cast<char*>(staging), unpack ? 1 : 0);
    return check_launch("strided_pack");
}
