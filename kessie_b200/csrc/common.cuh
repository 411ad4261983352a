// common.cuh -- shared host/device helpers for libkessie_cuda.so (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stddef.h>

#include "../../include/kessie_capi.h"

#include <nvtx3/nvToolsExt.h>

namespace kessie {

// ---------------------------------------------------------------- host errors
// Record a status + message for kessie_get_last_error(); returns `code`.
int set_error(int code, const char* fmt, ...);
// Clear the calling thread's error (successful call).
void clear_error();
// Map a CUDA error after a launch to a status; returns 0 when none.
int check_launch(const char* what);

// Device address of this library's status word on the current device.
int* device_status_ptr();
// Number of SMs of the current device (cached per device).
int sm_count();

// ------------------------------------------- programmatic dependent launches
// Kernels of this library launched as programmatic dependents wait for the
// preceding grid (griddepcontrol.wait) before they let the next launch start
// (launch_dependents), so while one runs, at most its immediate predecessor
// still runs.  Such a kernel may issue loads before its wait ("early reads")
// when that predecessor writes none of the bytes the loads read.  The
// library records, per (device, stream), the byte ranges written by the last
// programmatic launch it made there; a launch that is not programmatic
// (library or not) serialises fully and needs no record.
struct ByteRange { uintptr_t lo, hi; };
// Holds the registry locked from a claim until the launch it decided has
// been issued, so the record follows the stream's real launch order when
// several host threads launch on one stream.
class LaunchOrderGuard {
  public:
    LaunchOrderGuard();
    ~LaunchOrderGuard();
    LaunchOrderGuard(const LaunchOrderGuard&) = delete;
    LaunchOrderGuard& operator=(const LaunchOrderGuard&) = delete;
};
// Records `writes` as the last programmatic launch on (current device,
// `stream`) and returns true when none of the previous record's ranges
// overlaps any of `reads` (an empty range overlaps nothing).  The caller
// holds a LaunchOrderGuard from before this call until its launch is issued.
//
// Every launch of this library signals its dependents only after its own
// griddepcontrol.wait, except the context-parallel combine, which signals at
// its start (so the next step's decode overlaps this step's tail) and waits
// for the decode at its end.  Such a launch passes `merge` (its record keeps
// the previous record's writes: that launch may still run when the next one
// starts) and `delay_ns`, a bound on how long its dependents can sit in
// griddepcontrol.wait after it signalled (its cross-rank wait).  A caller
// that gives no `prev_delay_ns` gets false after such a launch, since its
// bounded waits do not cover that delay; one that does gets the delay, to add
// to every bounded wait that may sit behind another thread's
// griddepcontrol.wait.
bool claim_early_reads(cudaStream_t stream, const ByteRange* reads, int nreads, const ByteRange* writes,
                       int nwrites, uint64_t* prev_delay_ns = nullptr, uint64_t delay_ns = 0, bool merge = false);
// [p, p + bytes) as a byte range (empty for a null pointer or no bytes).
inline ByteRange byte_span(const void* p, int64_t bytes) {
    const uintptr_t b = reinterpret_cast<uintptr_t>(p);
    return (p && bytes > 0) ? ByteRange{b, b + (uintptr_t)bytes} : ByteRange{0, 0};
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Scoped NVTX range around a C-ABI entry point, so host-side timelines
// (Nsight Systems, or any NVTX tool) show which library call launched what.
// Header-only NVTX: without an attached tool each push / pop is one test of a
// function pointer.
class NvtxRange {
  public:
    explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange&) = delete;
    NvtxRange& operator=(const NvtxRange&) = delete;
};

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// ---------------------------------------------------------------- dtypes
template <int DT> struct Elem;
template <> struct Elem<KESSIE_DTYPE_F16>  { using T = __half;        static constexpr int bytes = 2; };
template <> struct Elem<KESSIE_DTYPE_BF16> { using T = __nv_bfloat16; static constexpr int bytes = 2; };
template <> struct Elem<KESSIE_DTYPE_F32>  { using T = float;         static constexpr int bytes = 4; };

inline int dtype_bytes(int dt) { return dt == KESSIE_DTYPE_F32 ? 4 : 2; }
inline bool dtype_ok(int dt) { return dt == KESSIE_DTYPE_F16 || dt == KESSIE_DTYPE_BF16 || dt == KESSIE_DTYPE_F32; }

__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f32(float x) { return x; }
template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }

// 16-byte vector of elements: 8 halves / 8 bf16 / 4 floats.
template <typename T> struct Vec16 { static constexpr int N = 16 / sizeof(T); };

__device__ __forceinline__ void record_status(int* status, int bits) {
    if (status) atomicOr(status, bits);
}

// Streaming 16-byte global load that does not allocate in L1.
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}
__device__ __forceinline__ float4 ldg_stream_f4(const float* p) {
    float4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w) : "l"(p));
    return r;
}
__device__ __forceinline__ void stg_stream(void* p, uint4 v) {
    asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};"
                 :: "l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}

// 16-byte asynchronous copy global -> shared (cached in L2 only): the bytes in
// flight occupy shared memory, not registers.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(d), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
// Wait until at most N of this thread's most recent cp.async groups are pending.
template <int N>
__device__ __forceinline__ void cp_async_wait_group() { asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory"); }

}  // namespace kessie
