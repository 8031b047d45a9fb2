// m3_mimo_step_static: the single-launch decode step with scratch memory
// that belongs to the library instead of the caller.
//
// m3_mimo_step needs a device workspace from its caller (the in_proj output,
// the gated output and the grid-barrier words live there).  Some callers
// cannot provide one: a plugin that is handed device buffers by a host
// framework but has no access to that framework's allocator, a serving
// thread that must never call cudaMalloc (it can synchronise the device and
// take milliseconds), or a process whose device footprint is fixed after
// start-up.  This entry point serves them from a file-scope device array of
// kStaticScratchBytes that every GPU loading the library holds until the
// process exits.  It allocates nothing itself and calls no allocating
// routine.
//
// The array is shared by every call on a device and keeps the last call's
// contents; the barrier words that a launch needs at zero are cleared on the
// caller's stream before each launch.  Calls that overlap on the GPU (on
// different streams, or from different threads) race on the array.
#include <cstdint>
#include <mutex>

#include "m3_step.cuh"

namespace {

constexpr int64_t kStaticScratchBytes = M3_STEP_STATIC_SCRATCH_BYTES;
static_assert(kStaticScratchBytes % 256 == 0, "scratch size must keep 256-byte alignment");

static __device__ __align__(256) unsigned char g_step_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void *g_scratch_addr[kMaxDevices] = {nullptr};

// Device address of the scratch array on the current device.  The array's
// name is only a host-side handle, so the address is looked up once per
// device (with that device current) and cached.
int scratch_address(void **addr) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return M3_ERR_DEVICE;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_addr[dev] == nullptr) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_step_scratch) != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return M3_ERR_DEVICE;
    }
    g_scratch_addr[dev] = p;
  }
  *addr = g_scratch_addr[dev];
  return M3_OK;
}

}  // namespace

extern "C" int m3_mimo_step_static(const m3_dims *dims, const m3_step_args *args, m3_stream_t stream) {
  if (!dims || !args) return M3_ERR_NULL;
  if (args->workspace != nullptr || args->workspace_bytes != 0) return M3_ERR_SHAPE;
  const int64_t need = m3_mimo_step_workspace_bytes(dims, args->d_model, args->dtype);
  if (need < 0) return (int)-need;
  if (need > kStaticScratchBytes) return M3_ERR_SCRATCH;
  void *scratch = nullptr;
  const int st = scratch_address(&scratch);
  if (st != M3_OK) return st;
  m3_step_args a = *args;
  a.workspace = scratch;
  a.workspace_bytes = kStaticScratchBytes;
  // a call that m3_mimo_step would reject, or that has no rows, enqueues
  // nothing (and leaves the array alone)
  bool empty = false;
  const int check = m3::step_validate(dims, &a, &empty);
  if (check != M3_OK || empty) return check;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // the grid-barrier words start every call at zero
  if (cudaMemsetAsync(scratch, 0, m3::kStepBarBytes, s) != cudaSuccess) {
    cudaGetLastError();
    return M3_ERR_LAUNCH;
  }
  return m3_mimo_step(dims, &a, stream);
}
