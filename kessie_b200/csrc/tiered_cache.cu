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
    int B, H, T, chunks;          // chunks = row bytes / 16
    long long S;                  // live tokens after the append
    int fc, alpha_mode;
    float den, alpha;
};

template <typename T>
__global__ void __launch_bounds__(256) tiered_update_kernel(TieredUpdateArgs a) {
    const long long row_bytes = (long long)a.chunks * 16;
    const long long BH = (long long)a.B * a.H;
    const long long s_old = a.hi - a.lo;
    const long long v_rows = a.v_fog ? BH * a.S : BH * a.T;
    const long long total = (v_rows + BH * a.T) * a.chunks;
    for (long long it = blockIdx.x * (long long)blockDim.x + threadIdx.x; it < total;
         it += (long long)gridDim.x * blockDim.x) {
        const long long row = it / a.chunks;
        const int c = (int)(it - row * a.chunks);
        if (row < v_rows) {
            if (a.v_fog) {                                   // fogged V of the live range (+ V append)
                const long long bh = row / a.S, s = row - bh * a.S;
                const float w = tiered_fog_weight(s, a.fc, a.den, a.alpha, a.alpha_mode);
                uint4 raw;
                if (s < s_old) {
                    raw = ldg_stream(a.v_store + ((bh * a.cap + a.lo + s) * row_bytes + c * 16));
                } else {
                    const long long t = s - s_old, b = bh / a.H, h = bh - b * a.H;
                    raw = ldg_stream(a.v_new + (b * a.nsb + h * a.nsh + t * a.nst + c * 16));
                    *reinterpret_cast<uint4*>(a.v_store + ((bh * a.cap + a.hi + t) * row_bytes + c * 16)) = raw;
                }
                stg_stream(a.v_fog + (row * row_bytes + c * 16), scale16<T>(raw, w));
            } else {                                         // V append only
                const long long bh = row / a.T, t = row - bh * a.T, b = bh / a.H, h = bh - b * a.H;
                const uint4 raw = ldg_stream(a.v_new + (b * a.nsb + h * a.nsh + t * a.nst + c * 16));
                *reinterpret_cast<uint4*>(a.v_store + ((bh * a.cap + a.hi + t) * row_bytes + c * 16)) = raw;
            }
        } else {                                             // K append
            const long long r = row - v_rows;
            const long long bh = r / a.T, t = r - bh * a.T, b = bh / a.H, h = bh - b * a.H;
            const uint4 raw = ldg_stream(a.k_new + (b * a.nsb + h * a.nsh + t * a.nst + c * 16));
            *reinterpret_cast<uint4*>(a.k_store + ((bh * a.cap + a.hi + t) * row_bytes + c * 16)) = raw;
        }
    }
}

// Pack (unpack = 0) or unpack (1) tokens [t0, t0 + n) of M strided stores.
__global__ void __launch_bounds__(256) strided_pack_kernel(const unsigned long long* __restrict__ bases,
                                                           const long long* __restrict__ pitches, int M, long long BH,
                                                           long long n, int chunks, char* __restrict__ staging,
                                                           int unpack) {
    const long long row_bytes = (long long)chunks * 16;
    const long long total = (long long)M * BH * n * chunks;
    for (long long it = blockIdx.x * (long long)blockDim.x + threadIdx.x; it < total;
         it += (long long)gridDim.x * blockDim.x) {
        const long long row = it / chunks;
        const int c = (int)(it - row * chunks);
        const long long t = row % n, mb = row / n;
        const long long bh = mb % BH;
        const int m = (int)(mb / BH);
        char* store = reinterpret_cast<char*>(bases[m]) + bh * pitches[m] + t * row_bytes + c * 16;
        char* stage = staging + row * row_bytes + c * 16;
        if (unpack) *reinterpret_cast<uint4*>(store) = ldg_stream(stage);
        else stg_stream(stage, *reinterpret_cast<const uint4*>(store));
    }
}

int copy_grid(long long items) {
    const long long per = 256LL * 8;                       // 8 items per thread before the stride
    long long g = (items + per - 1) / per;
    const long long cap = (long long)sm_count() * 8;
    return (int)(g < 1 ? 1 : (g > cap ? cap : g));
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace kessie

using namespace kessie;

extern "C" int kessie_tiered_update_v2(void* k_store, void* v_store, long long cap, long long lo, long long hi,
                                       const void* k_new, const void* v_new, long long new_stride_b,
                                       long long new_stride_h, long long new_stride_t, int B, int H, int T, int D,
                                       int dtype, void* v_fog, float fog_alpha, double fog_start, void* stream) {
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
    TieredUpdateArgs a;
    a.k_store = static_cast<char*>(k_store);
    a.v_store = static_cast<char*>(v_store);
    a.k_new = static_cast<const char*>(k_new);
    a.v_new = static_cast<const char*>(v_new);
    a.v_fog = static_cast<char*>(v_fog);
    a.cap = cap; a.lo = lo; a.hi = hi;
    a.nsb = new_stride_b * es; a.nsh = new_stride_h * es; a.nst = new_stride_t * es;
    a.B = B; a.H = H; a.T = T; a.chunks = D * es / 16;
    a.S = S;
    a.fc = fc;
    a.den = (float)(fc - 1 > 1 ? fc - 1 : 1);
    a.alpha = fog_alpha;
    a.alpha_mode = fog_alpha == 0.5f ? 1 : fog_alpha == 1.f ? 2 : fog_alpha == 2.f ? 3 : fog_alpha == 3.f ? 4 : 0;
    const long long BH = (long long)B * H;
    const long long items = ((v_fog ? BH * S : BH * T) + BH * T) * a.chunks;
    if (items == 0) { clear_error(); return 0; }
    cudaStream_t st = as_stream(stream);
    const int grid = copy_grid(items);
    if (dtype == KESSIE_DTYPE_BF16) tiered_update_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(a);
    else if (dtype == KESSIE_DTYPE_F16) tiered_update_kernel<__half><<<grid, 256, 0, st>>>(a);
    else tiered_update_kernel<float><<<grid, 256, 0, st>>>(a);
    return check_launch("tiered_update");
}

extern "C" int kessie_strided_pack_v2(const unsigned long long* store_bases, const long long* store_pitch_bytes,
                                      int num_stores, int rows_per_store, long long tokens, int row_bytes,
                                      void* staging, int unpack, void* stream) {
    if (!store_bases || !store_pitch_bytes || !staging || num_stores <= 0 || rows_per_store <= 0 || tokens < 0 ||
        row_bytes <= 0 || row_bytes % 16 || !al16(staging))
        return set_error(KESSIE_ERR_ARG, "strided_pack_v2: bad arguments (row_bytes % 16 == 0, aligned staging)");
    const long long items = (long long)num_stores * rows_per_store * tokens * (row_bytes / 16);
    if (items == 0) { clear_error(); return 0; }
    strided_pack_kernel<<<copy_grid(items), 256, 0, as_stream(stream)>>>(
        store_bases, store_pitch_bytes, num_stores, rows_per_store, tokens, row_bytes / 16,
        static_cast<char*>(staging), unpack ? 1 : 0);
    return check_launch("strided_pack");
}
