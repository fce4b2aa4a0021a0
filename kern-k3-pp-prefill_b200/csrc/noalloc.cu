// k3moe_route_tables_noalloc: the routing-table builder for callers that may
// not allocate device memory.
//
// k3moe_route_tables needs a small scratch buffer (per-256-row-block expert
// counts and their running offsets) that the caller normally passes in.  Some
// callers cannot produce one: a host runtime that owns every device buffer and
// binds a fixed list of them to each call (a manifest executor, say), or a
// latency-critical loop where a cudaMalloc, which may synchronise the whole
// device, is not acceptable.  This entry keeps that scratch in a fixed array
// compiled into the library instead, so the call allocates nothing; the caller
// still passes the input ids and every output table.
//
// Limits and sharing: the array holds the scratch of at most
// K3MOE_NOALLOC_MAX_ROWS rows and K3MOE_NOALLOC_MAX_EXPERTS local experts
// (shared expert included) -- 513 KB, held on every GPU that loads the library
// until the process exits.  Larger calls are refused with K3MOE_ELIMIT.  All
// calls on a device use the same array: two calls whose work overlaps on the
// GPU (different streams, no ordering between them) race on it and produce
// wrong tables.  Every scratch word is written before it is read within a call,
// so nothing needs clearing between calls.  The first call on each device looks
// the array's device address up (cudaGetSymbolAddress, with that device
// current); make that first call before any stream capture.
#include <mutex>

namespace {

constexpr int kNoAllocMaxRows = K3MOE_NOALLOC_MAX_ROWS;
constexpr int kNoAllocMaxExperts = K3MOE_NOALLOC_MAX_EXPERTS;
// two [blocks][experts] int tables, each rounded up to 256 bytes (k3moe_route_scratch_bytes)
constexpr size_t kNoAllocScratchBytes =
    2 * (((size_t)(kNoAllocMaxRows / 256) * kNoAllocMaxExperts * 4 + 255) / 256 * 256);

// In host code this name is only a stand-in for the device array, never a
// device address: the kernel gets the address cudaGetSymbolAddress returns.
static __device__ __align__(256) unsigned char g_route_scratch[kNoAllocScratchBytes];

// Device address of g_route_scratch on the current device, looked up once per device.
int route_scratch_address(void** out) {
  static std::mutex mu;
  static void* addr[kMaxDevices] = {};
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return K3MOE_EINVAL;
  std::lock_guard<std::mutex> g(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_route_scratch) != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return K3MOE_ELAUNCH;
    }
    addr[dev] = p;
  }
  *out = addr[dev];
  return K3MOE_OK;
}

}  // namespace

extern "C" int k3moe_route_tables_noalloc(const int32_t* idx, int R, int K, int first, int E, int shared, int tile,
                                          int32_t* counts, int32_t* cta_batch, int32_t* cta_limit, int32_t* meta,
                                          int32_t* route_map, int32_t* exp2perm, k3moe_stream_t stream) {
  const int EL = E + (shared ? 1 : 0);
  if (R > kNoAllocMaxRows || EL > kNoAllocMaxExperts) return K3MOE_ELIMIT;
  if (R < 1 || E < 1) return K3MOE_EINVAL;
  if (k3moe_route_scratch_bytes(R, E, shared) > kNoAllocScratchBytes) return K3MOE_ELIMIT;
  void* scratch = nullptr;
  const int rc = route_scratch_address(&scratch);
  if (rc) return rc;
  return k3moe_route_tables(idx, R, K, first, E, shared, tile, scratch, counts, cta_batch, cta_limit, meta, route_map,
                            exp2perm, stream);
}
