// cp_exchange.cu -- exchange buffers of the context-parallel decode.
//
// Each rank allocates one buffer (layout in cp_layout.cuh) with cudaMalloc,
// exports it as a CUDA IPC handle, and maps the handles of the other ranks
// of its node.  The decode kernel stores its merged shard rows into every
// rank's buffer over NVLink (plain peer stores of self-validating words, no
// multicast); each rank's combine kernel reads only its own buffer.  The
// handles travel through the caller's process group (64 opaque bytes).
#include "common.cuh"
#include "cp_layout.cuh"

#include <string.h>

static_assert(sizeof(cudaIpcMemHandle_t) == KESSIE_IPC_HANDLE_BYTES, "IPC handle size");

using namespace kessie;

extern "C" int kessie_cp_exchange_alloc(size_t bytes, void** dev_ptr, void* ipc_handle) {
    if (!dev_ptr || !ipc_handle || bytes == 0) return set_error(KESSIE_ERR_ARG, "cp_exchange_alloc: bad arguments");
    *dev_ptr = nullptr;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) return set_error(KESSIE_ERR_CUDA, "cp_exchange_alloc: cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
    e = cudaMemset(p, 0, bytes);                         // flags start below every epoch (epochs are >= 1)
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return set_error(KESSIE_ERR_CUDA, "cp_exchange_alloc: %s", cudaGetErrorString(e));
    }
    memcpy(ipc_handle, &h, sizeof(h));
    *dev_ptr = p;
    clear_error();
    return KESSIE_OK;
}

extern "C" int kessie_cp_exchange_open(const void* ipc_handle, void** dev_ptr) {
    if (!dev_ptr || !ipc_handle) return set_error(KESSIE_ERR_ARG, "cp_exchange_open: bad arguments");
    *dev_ptr = nullptr;
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof(h));
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return set_error(KESSIE_ERR_CUDA, "cp_exchange_open: %s", cudaGetErrorString(e));
    *dev_ptr = p;
    clear_error();
    return KESSIE_OK;
}

extern "C" int kessie_cp_exchange_close(void* dev_ptr) {
    if (!dev_ptr) return set_error(KESSIE_ERR_ARG, "cp_exchange_close: null pointer");
    cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
    if (e != cudaSuccess) return set_error(KESSIE_ERR_CUDA, "cp_exchange_close: %s", cudaGetErrorString(e));
    clear_error();
    return KESSIE_OK;
}

extern "C" int kessie_cp_exchange_free(void* dev_ptr) {
    if (!dev_ptr) return set_error(KESSIE_ERR_ARG, "cp_exchange_free: null pointer");
    cudaError_t e = cudaFree(dev_ptr);
    if (e != cudaSuccess) return set_error(KESSIE_ERR_CUDA, "cp_exchange_free: %s", cudaGetErrorString(e));
    clear_error();
    return KESSIE_OK;
}
