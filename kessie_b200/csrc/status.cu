// status.cu -- last-error bookkeeping, device status word, device queries.
#include "common.cuh"

#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <map>
#include <mutex>
#include <utility>
#include <vector>

namespace {

thread_local char g_msg[512] = {0};
thread_local int g_status = 0;

// One status word per device context; OR of KESSIE_DEV_* bits.
__device__ int g_device_status;

constexpr int kMaxDevices = 64;
int* g_status_ptr[kMaxDevices] = {nullptr};
int g_sm_count[kMaxDevices] = {0};
std::mutex g_mu;

}  // namespace

namespace kessie {

int set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
    va_end(ap);
    g_status = code;
    return code;
}

void clear_error() {
    g_status = 0;
    g_msg[0] = 0;
}

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(KESSIE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    clear_error();
    return KESSIE_OK;
}

// Device address of the status word on the current device, looked up once per
// device and cached for the life of the process (a cudaDeviceReset of the
// device would leave it stale; the library is not used across one).
int* device_status_ptr() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_status_ptr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_device_status) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        g_status_ptr[dev] = static_cast<int*>(p);
    }
    return g_status_ptr[dev];
}

int sm_count() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_sm_count[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = 148;
        }
        g_sm_count[dev] = n;
    }
    return g_sm_count[dev];
}

namespace {
constexpr int kMaxWrites = 8;
struct LaunchWrites { int n; ByteRange r[kMaxWrites]; uint64_t delay_ns; };
std::mutex g_pdl_mu;
std::map<std::pair<int, uintptr_t>, LaunchWrites> g_last_pdl;
bool overlaps(const ByteRange& a, const ByteRange& b) { return a.lo < a.hi && b.lo < b.hi && a.lo < b.hi && b.lo < a.hi; }
}  // namespace

LaunchOrderGuard::LaunchOrderGuard() { g_pdl_mu.lock(); }
LaunchOrderGuard::~LaunchOrderGuard() { g_pdl_mu.unlock(); }

bool claim_early_reads(cudaStream_t stream, const ByteRange* reads, int nreads, const ByteRange* writes,
                       int nwrites, uint64_t* prev_delay_ns, uint64_t delay_ns, bool merge) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        dev = -1;
    }
    const auto key = std::make_pair(dev, reinterpret_cast<uintptr_t>(stream));
    auto it = g_last_pdl.find(key);
    const LaunchWrites* prev = it != g_last_pdl.end() ? &it->second : nullptr;
    bool early = true;
    if (prev)
        for (int i = 0; i < prev->n; ++i)
            for (int j = 0; j < nreads; ++j)
                if (overlaps(prev->r[i], reads[j])) early = false;
    const uint64_t pd = prev ? prev->delay_ns : 0;
    if (prev_delay_ns) *prev_delay_ns = pd;
    else if (pd) early = false;
    LaunchWrites w{};
    bool known = true;
    auto add = [&](const ByteRange& r) {
        if (r.lo >= r.hi) return;
        if (w.n == kMaxWrites) known = false;
        else w.r[w.n++] = r;
    };
    for (int i = 0; i < nwrites; ++i) add(writes[i]);
    w.delay_ns = delay_ns;
    if (merge && prev) {
        for (int i = 0; i < prev->n; ++i) add(prev->r[i]);
        w.delay_ns = delay_ns + pd < delay_ns ? ~uint64_t(0) : delay_ns + pd;
    }
    if (!known) {
        early = false;
        w.n = 1;                                    // unknown writes: everything overlaps the next reads
        w.r[0] = ByteRange{0, ~uintptr_t(0)};
    }
    g_last_pdl[key] = w;
    return early;
}

}  // namespace kessie

extern "C" int kessie_get_last_error(char* buf, int len) {
    if (buf && len > 0) {
        strncpy(buf, g_msg, (size_t)len - 1);
        buf[len - 1] = 0;
    }
    return g_status;
}

extern "C" const char* kessie_version(void) { return "kessie_b200 0.1 sm_100a"; }

extern "C" int kessie_launch_registry_claim(void* stream, const uint64_t* reads, int nreads, const uint64_t* writes,
                                            int nwrites, uint64_t delay_ns, int merge, uint64_t* prev_delay_ns,
                                            int* may_read_early) {
    using namespace kessie;
    if (!may_read_early || nreads < 0 || nwrites < 0 || nreads > 4096 || nwrites > 4096 || (nreads && !reads) ||
        (nwrites && !writes))
        return set_error(KESSIE_ERR_ARG, "launch_registry_claim: bad range arrays");
    std::vector<ByteRange> r((size_t)nreads), w((size_t)nwrites);
    for (int i = 0; i < nreads; ++i) r[i] = ByteRange{(uintptr_t)reads[2 * i], (uintptr_t)reads[2 * i + 1]};
    for (int i = 0; i < nwrites; ++i) w[i] = ByteRange{(uintptr_t)writes[2 * i], (uintptr_t)writes[2 * i + 1]};
    LaunchOrderGuard order;
    *may_read_early = claim_early_reads(as_stream(stream), r.data(), nreads, w.data(), nwrites, prev_delay_ns,
                                        delay_ns, merge != 0) ? 1 : 0;
    clear_error();
    return KESSIE_OK;
}

extern "C" int kessie_read_device_status(void* stream) {
    int* p = kessie::device_status_ptr();
    if (!p) return kessie::set_error(KESSIE_ERR_CUDA, "device status word unavailable");
    cudaStream_t s = kessie::as_stream(stream);
    int host = 0;
    if (cudaMemcpyAsync(&host, p, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaMemsetAsync(p, 0, sizeof(int), s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess) {
        cudaError_t e = cudaGetLastError();
        return kessie::set_error(KESSIE_ERR_CUDA, "read_device_status: %s", cudaGetErrorString(e));
    }
    kessie::clear_error();
    return host;
}
