// Library-wide C ABI pieces: error reporting, the device error word, device
// properties.  The per-operator entry points live beside their kernels.
#include <atomic>
#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"

namespace gorgon {

namespace {
thread_local std::string g_last_error;

// One 32-bit error word per device; kernels OR error bits into it.
__device__ uint32_t g_device_error_word;

constexpr int kMaxDevices = 64;
std::mutex g_dev_mu;
uint32_t* g_err_addr[kMaxDevices] = {};
int g_sm_count[kMaxDevices] = {};
std::atomic<uint64_t> g_wait_limit_ns{2000000000ull};
}  // namespace

uint64_t wait_limit_ns() { return g_wait_limit_ns.load(std::memory_order_relaxed); }

int set_error(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return GORGON_OK;
  return set_error(GORGON_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

uint32_t* device_error_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (!g_err_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error_word) != cudaSuccess) return nullptr;
    g_err_addr[dev] = static_cast<uint32_t*>(p);
  }
  return g_err_addr[dev];
}

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (!g_sm_count[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}

}  // namespace gorgon

extern "C" int gorgon_abi_version(void) { return GORGON_ABI_VERSION; }

extern "C" const char* gorgon_last_error(void) { return gorgon::g_last_error.c_str(); }

extern "C" int gorgon_device_error(uint32_t* out_flags, int clear) {
  using namespace gorgon;
  if (!out_flags) return set_error(GORGON_ERR_INVALID, "gorgon_device_error: out_flags is null");
  uint32_t v = 0;
  int rc = check_cuda(cudaMemcpyFromSymbol(&v, g_device_error_word, sizeof(v)), "read device error word");
  if (rc) return rc;
  *out_flags = v;
  if (clear) {
    uint32_t z = 0;
    rc = check_cuda(cudaMemcpyToSymbol(g_device_error_word, &z, sizeof(z)), "clear device error word");
    if (rc) return rc;
  }
  return GORGON_OK;
}

extern "C" int64_t gorgon_set_wait_limit_ns(int64_t ns) {
  using namespace gorgon;
  const uint64_t prev = g_wait_limit_ns.load();
  if (ns > 0) g_wait_limit_ns.store(static_cast<uint64_t>(ns));
  return static_cast<int64_t>(prev);
}

// ---- peer buffers for the fused output gather (CUDA IPC between the
// processes of one node; the mapping enables peer access over NVLink)
static_assert(sizeof(cudaIpcMemHandle_t) == sizeof(gorgon_ipc_handle), "IPC handle size");

extern "C" int gorgon_peer_buffer_alloc(size_t bytes, void** ptr, gorgon_ipc_handle* handle) {
  using namespace gorgon;
  if (!ptr || !handle || bytes == 0) return set_error(GORGON_ERR_INVALID, "gorgon_peer_buffer_alloc: bad argument");
  void* p = nullptr;
  int rc = check_cuda(cudaMalloc(&p, bytes), "gorgon_peer_buffer_alloc: cudaMalloc");
  if (rc) return rc;
  rc = check_cuda(cudaMemset(p, 0, bytes), "gorgon_peer_buffer_alloc: cudaMemset");
  if (!rc) rc = check_cuda(cudaDeviceSynchronize(), "gorgon_peer_buffer_alloc: synchronize");
  if (!rc) {
    cudaIpcMemHandle_t h;
    rc = check_cuda(cudaIpcGetMemHandle(&h, p), "gorgon_peer_buffer_alloc: cudaIpcGetMemHandle");
    if (!rc) std::memcpy(handle->bytes, &h, sizeof(h));
  }
  if (rc) {
    cudaFree(p);
    return rc;
  }
  *ptr = p;
  return GORGON_OK;
}

extern "C" int gorgon_peer_buffer_open(const gorgon_ipc_handle* handle, void** ptr) {
  using namespace gorgon;
  if (!ptr || !handle) return set_error(GORGON_ERR_INVALID, "gorgon_peer_buffer_open: bad argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle->bytes, sizeof(h));
  return check_cuda(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "gorgon_peer_buffer_open: cudaIpcOpenMemHandle");
}

extern "C" int gorgon_peer_buffer_close(void* peer_ptr) {
  using namespace gorgon;
  if (!peer_ptr) return GORGON_OK;
  return check_cuda(cudaIpcCloseMemHandle(peer_ptr), "gorgon_peer_buffer_close: cudaIpcCloseMemHandle");
}

extern "C" int gorgon_peer_buffer_free(void* ptr) {
  using namespace gorgon;
  if (!ptr) return GORGON_OK;
  return check_cuda(cudaFree(ptr), "gorgon_peer_buffer_free: cudaFree");
}
