// Priority update for callers that cannot allocate device memory.
//
// per_update_priorities() needs device scratch beyond its inputs and outputs
// once a batch is too large for its partitioned path (more than 2048
// indices): one claim word per slot and per tree node, which elect the one
// writer of each slot and node, plus the words of a grid barrier. Its callers
// allocate that scratch themselves and pass it in per_store_t (claims[],
// scratch).
//
// Some callers cannot allocate: an application that hands this library a
// fixed device-memory budget at start-up and forbids any allocation
// afterwards (robotics and simulation runtimes often work this way), or code
// on a latency-critical path where cudaMalloc/cudaFree would synchronise the
// device. per_update_priorities_noalloc() serves them with scratch compiled
// into the library: a file-scope __device__ array, sized for stores of up to
// PER_NOALLOC_MAX_CAPACITY slots, which every GPU that loads the library holds
// until the process exits. The function itself calls no cudaMalloc,
// cudaFree or allocating library routine.
//
// Host code cannot use the array's name as a device address (on the host it
// is only a stand-in symbol), so the first call on each device, with that
// device current, resolves the address with cudaGetSymbolAddress and caches
// it. Make that first call before any stream capture.
//
// All calls share the one array and it keeps the previous call's contents.
// Batches of up to 2048 indices take the partitioned path, which uses none of
// it; a larger batch first clears, on its stream, the claim words and barrier
// words that its grid uses (a grid that gave up at a bounded wait may have
// left them set). Two calls whose work overlaps on the GPU (different streams,
// or different stores at the same time) race on the array: serialise them.
// The cached address belongs to the device's current context: after
// cudaDeviceReset() on a device, do not call this function there again.
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "per_b200.h"
#include "per_internal.h"

// The scratch array. Every GPU that loads the library holds it until exit.
static __device__ __align__(256) unsigned char per_noalloc_scratch[PER_NOALLOC_SCRATCH_BYTES];

namespace {

// Byte layout of the static scratch: the grid-barrier words, then the claim
// words of levels 0, 1 and 2 for a store of PER_NOALLOC_MAX_CAPACITY slots
// (stores up to that size have exactly three levels), each region 256-byte
// aligned.
constexpr int64_t kCap = PER_NOALLOC_MAX_CAPACITY;
constexpr size_t kAlign = 256;
constexpr size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }
constexpr size_t kOffBarrier = 0;
constexpr size_t kOffClaims0 = align_up(kOffBarrier + PER_SCRATCH_BYTES);
constexpr size_t kOffClaims1 = align_up(kOffClaims0 + 4 * (size_t)kCap);
constexpr size_t kOffClaims2 = align_up(kOffClaims1 + 4 * (size_t)(kCap / PER_FANOUT));
constexpr size_t kBytes = align_up(kOffClaims2 + 4 * (size_t)(kCap / PER_BLOCK_P + PER_FANOUT));
static_assert(kBytes == PER_NOALLOC_SCRATCH_BYTES, "stated scratch size");

constexpr int kMaxDevices = 64;
void* g_scratch[kMaxDevices];
std::mutex g_mu;

// Device address of the scratch array on the current device (set up once
// per device).
int scratch_address(unsigned char** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return per_record_cuda(e);
  if (dev < 0 || dev >= kMaxDevices) return PER_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, per_noalloc_scratch);
    if (e != cudaSuccess) return per_record_cuda(e);
    g_scratch[dev] = p;
  }
  *out = static_cast<unsigned char*>(g_scratch[dev]);
  return PER_OK;
}

}  // namespace

extern "C" int per_update_priorities_noalloc(const per_store_t* s, const int64_t* idx,
                                             const float* td, int64_t n, void* stream) {
  if (!s) return PER_ERR_NULL_POINTER;
  if (s->capacity > PER_NOALLOC_MAX_CAPACITY) return PER_ERR_TOO_LARGE;
  int rc = per_check_store(s, false);  // claims[] and scratch come from the array
  if (rc) return rc;
  if (s->num_levels != 3) return PER_ERR_INVALID_ARGUMENT;
  if (!idx || !td) return PER_ERR_NULL_POINTER;
  if (n < 1) return PER_ERR_EMPTY;
  if (n >= (int64_t)0xffffffffLL) return PER_ERR_TOO_LARGE;

  unsigned char* base = nullptr;
  rc = scratch_address(&base);
  if (rc) return rc;

  PerTree t = per_tree_of(s);
  for (int k = 0; k < PER_MAX_LEVELS; ++k) t.claims[k] = nullptr;
  t.claims[0] = reinterpret_cast<uint32_t*>(base + kOffClaims0);
  t.claims[1] = reinterpret_cast<uint32_t*>(base + kOffClaims1);
  t.claims[2] = reinterpret_cast<uint32_t*>(base + kOffClaims2);
  t.scratch = reinterpret_cast<PerScratch*>(base + kOffBarrier);

  // the partitioned path touches none of the array; the grid path starts from
  // cleared barrier and claim words (the previous call's contents stay)
  cudaStream_t st = (cudaStream_t)stream;
  if (per_update_uses_grid(t, n)) {
    cudaError_t e = cudaMemsetAsync(base + kOffBarrier, 0, PER_SCRATCH_BYTES, st);
    for (int k = 0; k < 3 && e == cudaSuccess; ++k)
      e = cudaMemsetAsync(t.claims[k], 0, (size_t)s->level_len[k] * 4, st);
    if (e != cudaSuccess) return per_record_cuda(e);
  }
  return per_launch_update(t, idx, td, n, st);
}
