// kessie_hip_binding.cpp -- the torch extension module `kessie_hip`: the
// reference's second boundary (kessie_hip_binding.cpp:216-239, a pybind11
// torch extension over the same five launchers), rebuilt over this library's
// C ABI.  Same module name, function names, argument names, defaults and
// input checks, so `import kessie_hip` code keeps working; kernels run on the
// current PyTorch CUDA stream, as the reference's run on the current HIP
// stream.  A launcher failure, which the reference cannot see, raises here.
//
// The launchers are resolved from libkessie_cuda.so, which the loader
// (kessie_b200._lib.load_binding) opens with RTLD_GLOBAL before importing this
// module.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include <cmath>

#include "../../include/kessie_capi.h"

namespace {

void* current_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

// The legacy launchers return void and record failures; surface them.
void raise_on_failure(const char* what) {
    char msg[512];
    const int st = kessie_get_last_error(msg, (int)sizeof(msg));
    TORCH_CHECK(st == 0, what, " failed: ", msg);
}

void check_attention_inputs(const torch::Tensor& Q, const torch::Tensor& K, const torch::Tensor& V) {
    TORCH_CHECK(Q.is_cuda(), "Q must be on GPU");
    TORCH_CHECK(Q.dtype() == torch::kHalf, "Q must be FP16");
    TORCH_CHECK(Q.is_contiguous() && K.is_contiguous() && V.is_contiguous(), "Q, K, V must be contiguous");
    TORCH_CHECK(K.sizes() == Q.sizes() && V.sizes() == Q.sizes(), "K and V must have Q's shape [B, H, N, D]");
    TORCH_CHECK(K.dtype() == Q.dtype() && V.dtype() == Q.dtype(), "K and V must be FP16 like Q");
    TORCH_CHECK(Q.dim() == 4, "Q must be [B, H, N, D]");
    TORCH_CHECK(Q.size(3) == 64 || Q.size(3) == 128, "head_dim must be 64 or 128");
}

torch::Tensor windowed_attention(torch::Tensor Q, torch::Tensor K, torch::Tensor V, int64_t window_size,
                                 bool causal) {
    check_attention_inputs(Q, K, V);
    const int B = (int)Q.size(0), H = (int)Q.size(1), N = (int)Q.size(2), D = (int)Q.size(3);
    auto O = torch::empty_like(Q);
    launch_kessie_windowed_attn(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(),
                                1.0f / std::sqrt((float)D), B, H, N, D, (int)window_size, causal ? 1 : 0,
                                current_stream());
    raise_on_failure("windowed_attention");
    return O;
}

torch::Tensor fused_fog_attention(torch::Tensor Q, torch::Tensor K, torch::Tensor V, torch::Tensor fog_weights,
                                  int64_t window_size, bool causal) {
    check_attention_inputs(Q, K, V);
    TORCH_CHECK(fog_weights.dtype() == torch::kFloat, "fog_weights must be FP32");
    TORCH_CHECK(fog_weights.is_cuda() && fog_weights.is_contiguous() && fog_weights.numel() == Q.size(2),
                "fog_weights must be a contiguous [N] tensor on the GPU");
    const int B = (int)Q.size(0), H = (int)Q.size(1), N = (int)Q.size(2), D = (int)Q.size(3);
    auto O = torch::empty_like(Q);
    launch_kessie_fused_fog_attn(Q.data_ptr(), K.data_ptr(), V.data_ptr(), O.data_ptr(), fog_weights.data_ptr(),
                                 1.0f / std::sqrt((float)D), B, H, N, D, (int)window_size, causal ? 1 : 0,
                                 current_stream());
    raise_on_failure("fused_fog_attention");
    return O;
}

void rope_remap(torch::Tensor k_data, torch::Tensor orig_positions, torch::Tensor target_positions,
                double rope_theta) {
    TORCH_CHECK(k_data.is_cuda(), "k_data must be on GPU");
    TORCH_CHECK(k_data.is_contiguous(), "k_data must be contiguous");
    TORCH_CHECK(k_data.dtype() == torch::kHalf, "k_data must be FP16");
    TORCH_CHECK(orig_positions.dtype() == torch::kInt && target_positions.dtype() == torch::kInt,
                "positions must be INT32");
    TORCH_CHECK(k_data.dim() == 3 && k_data.size(2) % 2 == 0, "k_data must be [tokens, heads, dim], dim even");
    launch_kessie_rope_remap(k_data.data_ptr(), orig_positions.data_ptr(), target_positions.data_ptr(),
                             (float)rope_theta, (int)k_data.size(0), (int)k_data.size(1), (int)(k_data.size(2) / 2),
                             current_stream());
    raise_on_failure("rope_remap");
}

torch::Tensor page_evict(torch::Tensor page_valid, torch::Tensor page_positions, int64_t evict_before_pos) {
    TORCH_CHECK(page_valid.is_cuda(), "page_valid must be on GPU");
    TORCH_CHECK(page_valid.dtype() == torch::kInt8, "page_valid must be int8");
    TORCH_CHECK(page_positions.dtype() == torch::kInt, "page_positions must be INT32");
    auto evict_count = torch::zeros({1}, torch::dtype(torch::kInt32).device(page_valid.device()));
    launch_kessie_page_evict(page_valid.data_ptr(), page_positions.data_ptr(), evict_count.data_ptr(),
                             (int)evict_before_pos, (int)page_valid.size(0), current_stream());
    raise_on_failure("page_evict");
    return evict_count;
}

void page_insert(torch::Tensor kv_cache, torch::Tensor new_keys, torch::Tensor new_values,
                 torch::Tensor target_page_ids, torch::Tensor page_valid, torch::Tensor page_positions,
                 int64_t insert_conv_position) {
    TORCH_CHECK(kv_cache.is_cuda(), "kv_cache must be on GPU");
    TORCH_CHECK(kv_cache.dtype() == torch::kHalf, "kv_cache must be FP16");
    TORCH_CHECK(kv_cache.dim() == 5, "kv_cache must be [pages, page_size, 2, heads, dim]");
    TORCH_CHECK(new_keys.dim() == 3 && new_values.sizes() == new_keys.sizes(),
                "new_keys / new_values must be [tokens, heads, dim]");
    TORCH_CHECK(target_page_ids.dtype() == torch::kInt, "target_page_ids must be INT32");
    launch_kessie_page_insert(kv_cache.data_ptr(), new_keys.data_ptr(), new_values.data_ptr(),
                              target_page_ids.data_ptr(), page_valid.data_ptr(), page_positions.data_ptr(),
                              (int)insert_conv_position, (int)new_keys.size(0), (int)new_keys.size(1),
                              (int)new_keys.size(2), (int)kv_cache.size(1), (int)kv_cache.size(0),
                              current_stream());
    raise_on_failure("page_insert");
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.doc() = "KeSSie fog attention, RoPE remap and page management on B200 (libkessie_cuda.so)";
    m.def("windowed_attention", &windowed_attention, "Windowed causal attention, FP16 [B, H, N, D]",
          py::arg("Q"), py::arg("K"), py::arg("V"), py::arg("window_size") = 0, py::arg("causal") = true);
    m.def("fused_fog_attention", &fused_fog_attention, "Attention with fog weights on V, FP16 [B, H, N, D]",
          py::arg("Q"), py::arg("K"), py::arg("V"), py::arg("fog_weights"), py::arg("window_size") = 0,
          py::arg("causal") = true);
    m.def("rope_remap", &rope_remap, "Re-rotate K from original to target positions, in place",
          py::arg("k_data"), py::arg("orig_positions"), py::arg("target_positions"),
          py::arg("rope_theta") = 10000.0);
    m.def("page_evict", &page_evict, "Mark valid pages below a position free; returns the count",
          py::arg("page_valid"), py::arg("page_positions"), py::arg("evict_before_pos"));
    m.def("page_insert", &page_insert, "Copy K/V tokens into target pages and mark them valid",
          py::arg("kv_cache"), py::arg("new_keys"), py::arg("new_values"), py::arg("target_page_ids"),
          py::arg("page_valid"), py::arg("page_positions"), py::arg("insert_conv_position"));
}
