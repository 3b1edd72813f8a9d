// status.cu -- library-wide runtime pieces: the device status word, SM-count
// cache, version and error strings.
//
// The reference reports failures only through return codes
// (src/kernel/gdn_state_update_ref.cu:214-258) and TORCH_CHECK
// (src/ops/gdn_op.cu:54-96).  Here kernels additionally record conditions that
// only the device can see (a bounded wait that gave up, a slot index out of
// range) in one 32-bit word per device, which the host reads on demand.
#include <atomic>
#include <mutex>

#include "../common.cuh"

namespace gdn {

// One status word per device that loads the library; kernels atomicOr bits in.
static __device__ uint32_t g_device_status;

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mu;
uint32_t* g_status_ptr[kMaxDevices] = {};
int g_sm_count[kMaxDevices] = {};
}  // namespace

uint32_t* device_status_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_status_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_status) != cudaSuccess) return nullptr;
    g_status_ptr[dev] = static_cast<uint32_t*>(p);
  }
  return g_status_ptr[dev];
}

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_sm_count[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}

namespace {
struct SmemOptIn {
  const void* func;
  int dev;
  int bytes;
};
constexpr int kMaxOptIns = 256;
SmemOptIn g_optins[kMaxOptIns];
int g_num_optins = 0;
}  // namespace

int allow_dynamic_smem(const void* func, int bytes) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return GDN_ERR_CUDA;
  // The table is searched and extended under the lock, and the attribute is
  // set while holding it, so concurrent first calls set it once and every
  // caller returns only after it is in place.
  std::lock_guard<std::mutex> lk(g_mu);
  for (int i = 0; i < g_num_optins; ++i)
    if (g_optins[i].func == func && g_optins[i].dev == dev && g_optins[i].bytes >= bytes) return GDN_OK;
  if (cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) {
    (void)cudaGetLastError();
    return GDN_ERR_CUDA;
  }
  if (g_num_optins < kMaxOptIns) g_optins[g_num_optins++] = {func, dev, bytes};
  return GDN_OK;
}

// Exercises the bounded mbarrier wait every kernel uses (common.cuh) on both
// of its exits: a phase that completes (one arrival) and a phase that nothing
// completes, which must give up after timeout_ns and record the timeout bit.
// result = {first wait returned true, second returned true, microseconds the
// second waited}.
__global__ void wait_selftest_kernel(uint64_t timeout_ns, int32_t* result) {
  __shared__ uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  fence_mbar_init();
  mbar_arrive(&bar);  // completes phase 0
  const bool done = mbar_wait_bounded(&bar, 0, timeout_ns);
  const uint64_t t0 = globaltimer_ns();
  const bool stuck = mbar_wait_bounded(&bar, 1, timeout_ns);  // phase 1 gets no arrival
  const uint64_t waited = globaltimer_ns() - t0;
  if (!stuck) atomicOr(&g_device_status, kStatusWaitTimeout);
  result[0] = done ? 1 : 0;
  result[1] = stuck ? 1 : 0;
  result[2] = (int32_t)(waited / 1000u);
}

}  // namespace gdn

extern "C" int gdn_b200_selftest_wait(uint32_t timeout_us, int32_t* result, cudaStream_t stream) {
  if (!result || timeout_us == 0 || timeout_us > 2000000u) return GDN_ERR_ARGS;
  gdn::wait_selftest_kernel<<<1, 32, 0, stream>>>((uint64_t)timeout_us * 1000u, result);
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_LAUNCH;
}

extern "C" int gdn_b200_device_status(uint32_t* status_out, int clear, cudaStream_t stream) {
  if (!status_out) return GDN_ERR_ARGS;
  uint32_t* p = gdn::device_status_ptr();
  if (!p) return GDN_ERR_CUDA;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return GDN_ERR_CUDA;
  if (cudaMemcpy(status_out, p, sizeof(uint32_t), cudaMemcpyDeviceToHost) != cudaSuccess) return GDN_ERR_CUDA;
  if (clear && cudaMemset(p, 0, sizeof(uint32_t)) != cudaSuccess) return GDN_ERR_CUDA;
  return GDN_OK;
}

extern "C" const char* gdn_b200_error_string(int code) {
  switch (code) {
    case GDN_OK: return "ok";
    case GDN_ERR_ARGS: return "invalid argument (null pointer or bad size)";
    case GDN_ERR_LAUNCH: return "kernel launch failed";
    case GDN_ERR_UNSUPPORTED: return "unsupported shape or mode";
    case GDN_ERR_ALIGN: return "pointer or stride not 16-byte aligned";
    case GDN_ERR_CUDA: return "CUDA runtime query failed";
    default: return "unknown status";
  }
}

extern "C" const char* gdn_b200_version(void) { return "gdn_b200 0.1.0 sm_100a"; }
