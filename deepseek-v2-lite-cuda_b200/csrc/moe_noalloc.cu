// Allocation-free token dispatch.
//
// ds_moe_dispatch needs a few megabytes of scratch (per-block expert histograms, per-block
// slot bases, the rank of every (token, pick)) that its caller normally allocates and passes
// in.  Some callers cannot allocate device memory on the path that calls us: a serving loop
// that must not touch the CUDA allocator between requests (allocation can synchronise the
// device and stall other streams), a host-language binding that only holds plain pointers and
// has no allocator of its own, or code that runs while other work is being captured into a
// CUDA graph, where allocating is not allowed.  ds_moe_dispatch_noalloc serves them: the
// scratch lives in one fixed array in this library's device memory, so a call needs nothing
// beyond the inputs and outputs the caller already owns.
//
// Limits and sharing rules:
//   * num_tokens <= DS_NOALLOC_MAX_TOKENS (65536), num_experts <= 64, top_k <= 8; larger
//     calls are rejected with DS_ERR_UNSUPPORTED before anything is launched.
//   * The array (2.5 MiB) is reserved on every GPU that loads this library, until the process
//     exits.
//   * All calls on a device share it and it keeps whatever the previous call left in it.
//     Nothing in it has to start at zero: every entry a call reads was written earlier in the
//     same call.  Two calls whose kernels may overlap on the GPU (different streams without an
//     ordering between them, or several host threads) race on the array and corrupt each
//     other's results; order such calls on one stream.
//   * The first call on each device looks up the array's device address (a one-time set-up
//     that may load this library's device code); make that first call before any stream
//     capture begins.
//   * The address used is the current device's, so the stream must belong to the current
//     device; a stream of another device is rejected with DS_ERR_UNSUPPORTED.
#include <mutex>

#include "kernels.cuh"

namespace ds {
namespace {

constexpr int kNoAllocMaxTokens = DS_NOALLOC_MAX_TOKENS;
constexpr int kNoAllocMaxBlocks = (kNoAllocMaxTokens + kRouteTokens - 1) / kRouteTokens;
constexpr size_t kHistInts = static_cast<size_t>(kNoAllocMaxBlocks) * kMaxExperts;
constexpr size_t kRankInts = static_cast<size_t>(kNoAllocMaxTokens) * kMaxTopK;
constexpr size_t kScratchInts = 2 * kHistInts + kRankInts;

// The scratch itself.  In host code this name is only a stand-in for the symbol; the usable
// device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) int32_t g_dispatch_scratch[kScratchInts];

constexpr int kMaxDevices = 64;
int32_t* g_scratch_addr[kMaxDevices] = {};
std::mutex g_scratch_mutex;

// Device address of the scratch on the current device; looked up once per device.
int scratch_for_current_device(int32_t** out) {
  int dev = 0;
  DS_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(DS_ERR_UNSUPPORTED, "device ordinal %d", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_addr[dev] == nullptr) {
    int32_t* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&ptr), g_dispatch_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(dispatch scratch)");
    if (ptr == nullptr) return fail(DS_ERR_CUDA, "dispatch scratch has no device address");
    g_scratch_addr[dev] = ptr;
  }
  *out = g_scratch_addr[dev];
  return DS_OK;
}

}  // namespace
}  // namespace ds

extern "C" {

int ds_moe_dispatch_noalloc(const void* input_bf16, const int32_t* topk_indices,
                            const float* topk_weights, const int32_t* expert_offsets,
                            void* dispatched_bf16, int32_t* token_map, float* dispatched_weights,
                            int num_tokens, int hidden_size, int num_experts, int top_k,
                            void* stream) {
  DS_REQUIRE(num_tokens >= 0, "moe_dispatch_noalloc: num_tokens must be >= 0");
  if (num_tokens > ds::kNoAllocMaxTokens)
    return ds::fail(DS_ERR_UNSUPPORTED,
                    "moe_dispatch_noalloc: num_tokens=%d exceeds the fixed scratch limit of %d "
                    "tokens; use ds_moe_dispatch with a caller-provided workspace",
                    num_tokens, ds::kNoAllocMaxTokens);
  DS_REQUIRE(hidden_size > 0 && hidden_size % 8 == 0,
             "hidden_size must be divisible by 8 for 128-bit vectorized access.");
  DS_REQUIRE(num_experts >= 1 && num_experts <= ds::kMaxExperts,
             "moe_dispatch_noalloc: num_experts must be in [1, 64]");
  DS_REQUIRE(top_k >= 1 && top_k <= ds::kMaxTopK, "moe_dispatch_noalloc: top_k must be in [1, 8]");
  if (num_tokens == 0) return DS_OK;
  DS_REQUIRE(input_bf16 && topk_indices && topk_weights && expert_offsets && dispatched_bf16 &&
                 token_map && dispatched_weights,
             "moe_dispatch_noalloc: null pointer");
  DS_REQUIRE(ds::aligned16(input_bf16) && ds::aligned16(dispatched_bf16),
             "moe_dispatch_noalloc: input/dispatched must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (s != nullptr) {
    int cur = 0, sdev = 0;
    DS_CUDA(cudaGetDevice(&cur));
    DS_CUDA(cudaStreamGetDevice(s, &sdev));
    if (sdev != cur)
      return ds::fail(DS_ERR_UNSUPPORTED,
                      "moe_dispatch_noalloc: the stream belongs to device %d but device %d is "
                      "current; make the stream's device current first",
                      sdev, cur);
  }
  int32_t* scratch = nullptr;
  DS_TRY(ds::scratch_for_current_device(&scratch));
  const int nblk = ds::route_blocks(num_tokens);
  int32_t* hist = scratch;
  int32_t* base = scratch + ds::kHistInts;
  int32_t* rank = scratch + 2 * ds::kHistInts;
  DS_TRY(ds::launch_rank(topk_indices, num_tokens, num_experts, top_k, hist, rank, s));
  DS_TRY(ds::launch_plan(hist, nblk, num_experts, expert_offsets, nullptr, nullptr, base, s));
  return ds::launch_scatter(input_bf16, num_tokens, hidden_size, num_experts, top_k,
                            topk_indices, topk_weights, base, rank, dispatched_bf16, token_map,
                            dispatched_weights, nullptr, num_tokens * top_k, s);
}

}  // extern "C"
