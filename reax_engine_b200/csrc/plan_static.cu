// plan_static.cu -- the routing-data plan (reaxmoe_plan) for callers that cannot allocate device memory.
//
// Some callers of this library run where cudaMalloc is off limits: a plugin's enqueue step inside an inference
// runtime that plans all device memory ahead of time and forbids allocation while it executes. reaxmoe_plan_static
// gives them the same routing data as reaxmoe_plan without a caller workspace: its scratch (per-segment expert
// histograms and their prefix sums, the status word its count kernel needs) lives in one file-scope __device__
// array of fixed size, which every GPU that loads this library holds until the process exits. It reports no device
// status: routed ids outside [0, experts) are skipped, as reaxmoe_plan skips them, but nothing tells the caller.
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"

namespace reaxmoe {

int set_error(int code, const char* msg);  // api.cu: records the text returned by reaxmoe_last_error
int check_problem_shape(const reaxmoe_problem* p);  // api.cu: the shape checks of every entry point

// Limits of the static scratch: at most kStaticMaxTokens tokens (all experts up to kMaxExperts).
constexpr int kStaticMaxTokens = 65536;
constexpr int kStaticMaxSegments = kStaticMaxTokens / kSegTokens;                       // 512
constexpr size_t kStaticSegBytes = (size_t)kStaticMaxSegments * kMaxExperts * 4;          // 512 KiB
constexpr int kTableStride = kMaxExperts + 8;                                           // E+1 entries, padded
constexpr size_t kStaticTableBytes = 4 * kTableStride * 4;                               // counts, eoff, boff, tiles
constexpr size_t kStaticScratchBytes = 256 + 2 * kStaticSegBytes + kStaticTableBytes;     // ~1 MiB + 4.3 KiB

// The scratch itself. In host code this name is only a host-side stand-in, never a device address: the host
// must use the address that cudaGetSymbolAddress returns for the current device.
static __device__ __align__(256) unsigned char g_plan_scratch[kStaticScratchBytes];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_static_mu;
void* g_static_addr[kMaxDevices] = {};

// Device address of g_plan_scratch on the current device, looked up once per device (the first call on a device).
int static_scratch(void** out, int* dev_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return REAXMOE_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (g_static_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_plan_scratch) != cudaSuccess || p == nullptr) return REAXMOE_ERR_CUDA;
    g_static_addr[dev] = p;
  }
  *out = g_static_addr[dev];
  *dev_out = dev;
  return 0;
}
}  // namespace

}  // namespace reaxmoe

using namespace reaxmoe;

extern "C" {

int reaxmoe_plan_static(const reaxmoe_problem* p, const int32_t* topk_ids, int32_t* expert_offsets,
                        int32_t* blockscale_offsets, int32_t* problem_sizes1, int32_t* problem_sizes2,
                        void* stream) {
  if (p == nullptr || topk_ids == nullptr || expert_offsets == nullptr || blockscale_offsets == nullptr)
    return set_error(REAXMOE_ERR_NULL, "plan_static: NULL pointer");
  const int rc = check_problem_shape(p);   // the same shape checks (and error text) as reaxmoe_plan
  if (rc) return rc;
  if (p->tokens > kStaticMaxTokens)
    return set_error(REAXMOE_ERR_BAD_SHAPE, "plan_static: tokens outside [0, 65536], the limit of its static scratch");
  void* base = nullptr;
  int dev = 0;
  if (static_scratch(&base, &dev) != 0)
    return set_error(REAXMOE_ERR_CUDA, "plan_static: cudaGetSymbolAddress of the static scratch failed");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* b = static_cast<uint8_t*>(base);
  int* status = reinterpret_cast<int*>(b);
  int* seg_counts = reinterpret_cast<int*>(b + 256);
  int* seg_base = reinterpret_cast<int*>(b + 256 + kStaticSegBytes);
  int* tables = reinterpret_cast<int*>(b + 256 + 2 * kStaticSegBytes);
  int* counts = tables;
  int* eoff = tables + kTableStride;
  int* boff = tables + 2 * kTableStride;
  int* tile_prefix = tables + 3 * kTableStride;
  const int nseg = (int)ceil_div64(p->tokens, kSegTokens);
  // The array keeps the previous call's contents: only the status word must start at zero; every other word
  // this call reads is written by this call first.
  if (cudaMemsetAsync(status, 0, sizeof(int), s) != cudaSuccess)
    return set_error(REAXMOE_ERR_CUDA, "plan_static: clearing the status word failed");
  if (p->tokens > 0) launch_count(topk_ids, p->tokens, p->topk, p->experts, seg_counts, status, s);
  launch_plan(seg_counts, nseg, p->experts, seg_base, counts, eoff, boff, tile_prefix, problem_sizes1,
              problem_sizes2, 2 * p->inter, p->hidden, p->hidden, p->inter, s);
  const size_t n = (size_t)(p->experts + 1) * 4;
  if (cudaMemcpyAsync(expert_offsets, eoff, n, cudaMemcpyDeviceToDevice, s) != cudaSuccess ||
      cudaMemcpyAsync(blockscale_offsets, boff, n, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
    return set_error(REAXMOE_ERR_CUDA, "plan_static: copying the offsets out failed");
  if (cudaPeekAtLastError() != cudaSuccess) return set_error(REAXMOE_ERR_CUDA, "plan_static: kernel launch failed");
  return REAXMOE_OK;
}

}  // extern "C"
