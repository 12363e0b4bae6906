// Library-wide host state: error messages, per-device facts and side streams, the device
// status word, the hello stub and the bounded-wait probe.
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "ptx.cuh"

namespace ds {

namespace {
thread_local char g_last_error[1024] = "";
constexpr int kMaxDevices = 64;
DeviceInfo g_info[kMaxDevices];
bool g_info_ready[kMaxDevices] = {};
std::mutex g_info_mutex;
}  // namespace

void set_last_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  snprintf(g_last_error, sizeof(g_last_error), "%s: %s (%s)", where, cudaGetErrorString(e),
           cudaGetErrorName(e));
  return DS_ERR_CUDA;
}

static SideStream g_side[kMaxDevices];
static bool g_side_ready[kMaxDevices] = {};
static std::mutex g_side_mutex;

int side_stream(int dev, SideStream* out) {
  if (dev < 0 || dev >= kMaxDevices) return fail(DS_ERR_UNSUPPORTED, "device ordinal %d", dev);
  std::lock_guard<std::mutex> lock(g_side_mutex);
  if (!g_side_ready[dev]) {
    SideStream ss{};
    DS_CUDA(cudaStreamCreateWithFlags(&ss.stream, cudaStreamNonBlocking));
    DS_CUDA(cudaEventCreateWithFlags(&ss.fork, cudaEventDisableTiming));
    DS_CUDA(cudaEventCreateWithFlags(&ss.join, cudaEventDisableTiming));
    g_side[dev] = ss;
    g_side_ready[dev] = true;
  }
  *out = g_side[dev];
  return DS_OK;
}

int device_info(DeviceInfo* out) {
  int dev = 0;
  DS_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(DS_ERR_UNSUPPORTED, "device ordinal %d", dev);
  std::lock_guard<std::mutex> lock(g_info_mutex);
  if (!g_info_ready[dev]) {
    DeviceInfo d{};
    d.device = dev;
    DS_CUDA(cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev));
    DS_CUDA(cudaDeviceGetAttribute(&d.clock_khz, cudaDevAttrClockRate, dev));
    if (d.clock_khz <= 0) d.clock_khz = 2000000;
    g_info[dev] = d;
    g_info_ready[dev] = true;
  }
  *out = g_info[dev];
  return DS_OK;
}

}  // namespace ds

// Status word written by kernels whose bounded waits ran out.
__device__ int g_ds_device_status;

namespace ds {
bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("DS_PDL");
    return e != nullptr && atoi(e) != 0;
  }();
  return on;
}

void add_pdl_attr(cudaLaunchAttribute* attrs, unsigned int& n) {
  if (!pdl_enabled()) return;
  attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[n].val.programmaticStreamSerializationAllowed = 1;
  ++n;
}

int* device_status_ptr() {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_ds_device_status) != cudaSuccess) return nullptr;
  return static_cast<int*>(p);
}
}  // namespace ds

namespace {

__global__ void hello_kernel() {
  if (threadIdx.x == 0) printf("Hello from ds_kernels on sm_100a (block %d)\n", blockIdx.x);
}

// One CTA; one thread waits on a barrier that nothing arrives on.
__global__ void wait_probe_kernel(int* status, long long timeout_cycles) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    ds::ptx::mbar_init(ds::ptx::smem_u32(&bar), 1);
    ds::ptx::fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    ds::ptx::mbar_wait(ds::ptx::smem_u32(&bar), 0, &abort_flag, status, timeout_cycles,
                       DS_ERR_TIMEOUT);
  }
  __syncwarp();
  __syncthreads();
}

}  // namespace

extern "C" {

const char* ds_last_error(void) { return ds::g_last_error; }

const char* ds_version(void) { return "ds_kernels sm_100a 0.1"; }

int ds_get_device_status(int* status) {
  DS_REQUIRE(status != nullptr, "ds_get_device_status: status is null");
  DS_CUDA(cudaDeviceSynchronize());
  int v = 0;
  DS_CUDA(cudaMemcpyFromSymbol(&v, g_ds_device_status, sizeof(int)));
  *status = v;
  return DS_OK;
}

int ds_clear_device_status(void) {
  int zero = 0;
  DS_CUDA(cudaDeviceSynchronize());
  DS_CUDA(cudaMemcpyToSymbol(g_ds_device_status, &zero, sizeof(int)));
  return DS_OK;
}

int ds_run_hello(void* stream) {
  hello_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>();
  DS_LAUNCH_CHECK("hello_kernel");
  return DS_OK;
}

int ds_debug_wait_probe(long long timeout_cycles, void* stream) {
  DS_REQUIRE(timeout_cycles > 0 && timeout_cycles <= (1LL << 34),
             "ds_debug_wait_probe: timeout_cycles must be in (0, 2^34]");
  int* status = ds::device_status_ptr();
  if (!status) return ds::fail(DS_ERR_CUDA, "device status word unavailable");
  wait_probe_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(status, timeout_cycles);
  DS_LAUNCH_CHECK("wait_probe_kernel");
  return DS_OK;
}

}  // extern "C"
