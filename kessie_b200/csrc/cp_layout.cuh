// cp_layout.cuh -- layout of the context-parallel exchange buffer.
//
// Every rank owns one exchange buffer in its own HBM; the other ranks of the
// node map it through CUDA IPC.  Rank r's decode stores its merged shard
// result for (seq b, q head h) into slot [par][r][b*Hq+h] of EVERY rank's
// buffer (plain stores over NVLink), and each rank's combine reads only its
// own buffer.
//
// Words are self-validating: every fp32 value travels in one 8-byte word
// together with the step's epoch, (value bits) | (epoch << 32), written with
// a single-copy-atomic 64-bit store.  A reader accepts a word once its high
// half equals the epoch it waits for, so no flag, fence or acquire is needed
// on either side and the decode never stalls on remote stores.
//
// par = epoch & 1 alternates between steps: rank A can only write slot par
// again in step e+2, which it reaches after its combine of step e+1, which
// needed rank B's words of step e+1, which B's decode wrote only after B's
// combine of step e finished reading slot par (stream order on B).
//
//   rows of (D + 2) words: D values of O/l, then m (log2 units), then l
//   [2 par][world src][B*Hq rows][D + 2]  (u64)
#pragma once

#include <stddef.h>
#include <stdint.h>

namespace kessie {

constexpr int kCpMaxRanks = 8;

struct CpLayout {
    int world, rows, D;
    __host__ __device__ size_t bytes() const {
        return ((size_t)2 * world * rows * (D + 2) * sizeof(uint64_t) + 255) & ~(size_t)255;
    }
    __host__ __device__ uint64_t* row(void* base, int par, int src, int r) const {
        return static_cast<uint64_t*>(base) + (((size_t)par * world + src) * rows + r) * (D + 2);
    }
};

__host__ __device__ __forceinline__ uint64_t cp_word(float v, uint32_t epoch) {
#ifdef __CUDA_ARCH__
    return (uint64_t)__float_as_uint(v) | ((uint64_t)epoch << 32);
#else
    union { float f; uint32_t u; } x{v};
    return (uint64_t)x.u | ((uint64_t)epoch << 32);
#endif
}

// Push targets of one decode launch: every rank's exchange buffer as mapped
// in this process (peer[rank] is this rank's own).  world == 0: no push.
struct CpLink {
    void* peer[kCpMaxRanks];
    int rank, world;
    uint32_t epoch;
};

}  // namespace kessie
