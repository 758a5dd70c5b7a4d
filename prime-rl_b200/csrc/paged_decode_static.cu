// Paged decode whose scratch memory is owned by the library, for callers that
// may not allocate device memory themselves.
//
// Who needs it: code that runs inside an inference engine which reserved the
// GPU's memory up front and hands none of it out to plugins.  vLLM, for
// example, sizes its KV cache to take most of HBM at start-up; a kernel library
// called from inside such an engine (a custom attention backend, an operator
// plugin) has no allocator it may use, and a late cudaMalloc of its own can fail
// or fragment what the engine reserved.  ps_paged_decode asks its caller for a
// workspace; this variant needs none.
//
// The scratch is a file-scope __device__ array of kStaticScratchBytes.  Every
// GPU that loads libps_attn.so holds one copy until the process exits.  In host
// code the array's name is only a stand-in symbol, never a device address: the
// device address is looked up with cudaGetSymbolAddress once per device (on the
// first call made with that device current) and cached.
#include <mutex>

#include "ps_attn.h"
#include "ps_common.cuh"
#include "ps_launch.h"

namespace {

constexpr int64_t kStaticScratchBytes = 16ll << 20;  // 16 MiB per GPU

__device__ __align__(256) uint8_t g_decode_scratch[kStaticScratchBytes];

// Device address of g_decode_scratch on the current device, looked up once per
// device.  Returns nullptr (and sets the message) on failure.
void* scratch_on_current_device() {
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    ps_set_last_error(PS_ERR_CUDA, "no usable current CUDA device");
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess || p == nullptr) {
      ps_set_last_error(PS_ERR_CUDA, "cudaGetSymbolAddress of the decode scratch array failed");
      return nullptr;
    }
    addr[dev] = p;
  }
  return addr[dev];
}

}  // namespace

extern "C" int ps_paged_decode_static_scratch(const ps_paged_problem* pr, void* stream) {
  if (pr == nullptr) return ps_paged_decode(pr, nullptr, 0, stream);  // reports the NULL problem
  if (pr->num_seqs <= 0) return ps_paged_decode(pr, nullptr, 0, stream);
  if (ps_paged_decode_workspace_size(pr->num_seqs, pr->num_q_heads, pr->num_kv_heads,
                                     pr->head_size) < 0)
    return PS_ERR_INVALID_ARGUMENT;  // message already set
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return ps_set_last_error(PS_ERR_CUDA, "no CUDA device");
  // the scratch this problem's kernel needs (16-bit and fp8 caches differ)
  const int64_t need = ps_decode_workspace_bytes(pr->num_seqs, pr->num_q_heads, pr->num_kv_heads, sms, 0,
                                                 pr->kv_cache_dtype == PS_KV_FP8_E4M3 ? 1 : 0);
  if (need > kStaticScratchBytes)
    return ps_set_last_error(PS_ERR_WORKSPACE,
                             "problem needs more decode scratch than the library's static 16 MiB "
                             "(fewer sequences per call, or ps_paged_decode with a workspace)");
  void* scratch = scratch_on_current_device();
  if (scratch == nullptr) return PS_ERR_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Calls share the array and it keeps the last call's contents.  The status
  // word and the per-(sequence, kv head) split counters must start at zero:
  // clear them (a completed call leaves the counters at zero, but a call that
  // gave up on a bounded wait may not).
  const size_t clear = 256 + static_cast<size_t>(pr->num_seqs) * pr->num_kv_heads * 4;
  if (cudaMemsetAsync(scratch, 0, clear, s) != cudaSuccess) return PS_ERR_CUDA;
  const int rc = ps_paged_decode(pr, scratch, kStaticScratchBytes, stream);
  if (rc != PS_OK) return rc;
  // hand this call's device status word to the caller's (optional) output
  if (pr->status != nullptr &&
      cudaMemcpyAsync(pr->status, scratch, sizeof(int32_t), cudaMemcpyDeviceToDevice, s) != cudaSuccess)
    return PS_ERR_CUDA;
  return PS_OK;
}
