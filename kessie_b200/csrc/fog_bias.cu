// fog_bias.cu -- builder of the reference's additive fog-bias buffer and the
// host conversion of the C-ABI description used by the attention entries.
#include "common.cuh"
#include "fog_bias.cuh"

namespace kessie {

int fog_bias_from_c(const kessie_fog_bias* in, FogBias* out) {
    *out = FogBias{};
    if (!in) return 0;
    if (in->recall_nbits < 0 || (in->recall_nbits > 0 && !in->recall_bits))
        return set_error(KESSIE_ERR_ARG, "fog bias: recall bitmap missing for %d bits", in->recall_nbits);
    if (in->dtype != KESSIE_DTYPE_F32 && in->dtype != KESSIE_DTYPE_BF16 && in->dtype != KESSIE_DTYPE_F16)
        return set_error(KESSIE_ERR_UNSUPPORTED, "fog bias: dtype %d", in->dtype);
    const bool fog = in->fog_alpha > 0.f;
    const bool recall = in->recall_bits && in->recall_nbits > 0;
    if (!fog && !recall) return 0;
    out->on = 1;
    out->keep = fog ? 1.0 - in->fog_start : 0.0;      // fb = 0 when fog_alpha <= 0: recall boost only
    out->neg_alpha = -in->fog_alpha;
    out->boost = in->recall_boost;
    out->recall = recall ? in->recall_bits : nullptr;
    out->recall_nbits = recall ? in->recall_nbits : 0;
    out->round_mode = in->dtype == KESSIE_DTYPE_BF16 ? 1 : (in->dtype == KESSIE_DTYPE_F16 ? 2 : 0);
    return 0;
}

namespace {

template <typename T>
__global__ void fog_bias_build_kernel(T* __restrict__ out, int kv_len, FogBias f) {
    const int fb = f.on ? fog_bias_boundary(f, kv_len) : 0;
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < kv_len; j += gridDim.x * blockDim.x)
        out[j] = from_f32<T>(f.on ? fog_bias_at(f, fb, j) : 0.f);
}

}  // namespace
}  // namespace kessie

using namespace kessie;

extern "C" int kessie_build_fog_bias_v2(void* out, int out_dtype, int kv_len, const kessie_fog_bias* bias,
                                        void* stream) {
    NvtxRange nvtx_range("kessie_build_fog_bias_v2");
    if (!out || kv_len < 0) return set_error(KESSIE_ERR_ARG, "build_fog_bias_v2: bad arguments");
    if (!dtype_ok(out_dtype)) return set_error(KESSIE_ERR_UNSUPPORTED, "build_fog_bias_v2: dtype %d", out_dtype);
    FogBias f;
    int rc = fog_bias_from_c(bias, &f);
    if (rc) return rc;
    if (kv_len == 0) { clear_error(); return 0; }
    const int threads = 256;
    const int blocks = (kv_len + threads - 1) / threads < 4096 ? (kv_len + threads - 1) / threads : 4096;
    cudaStream_t st = as_stream(stream);
    switch (out_dtype) {
        case KESSIE_DTYPE_F16: fog_bias_build_kernel<__half><<<blocks, threads, 0, st>>>((__half*)out, kv_len, f); break;
        case KESSIE_DTYPE_BF16: fog_bias_build_kernel<__nv_bfloat16><<<blocks, threads, 0, st>>>((__nv_bfloat16*)out, kv_len, f); break;
        default: fog_bias_build_kernel<float><<<blocks, threads, 0, st>>>((float*)out, kv_len, f); break;
    }
    return check_launch("build_fog_bias_v2");
}
