// cross_ntt_noalloc: the BAT NTT / INTT without any device allocation.
//
// Some callers cannot allocate device memory on their call path: a plugin
// loaded into a framework that has already reserved the GPU's memory for its
// own pool (JAX/XLA preallocates most of the device by default, so a
// cudaMalloc from the plugin can fail), or a latency-critical loop that
// cannot afford the device-wide synchronisation cudaFree implies.  For them
// this entry point takes only the input and output buffers; the NTT's
// intermediate (the step-1 result, batch * limbs * N words) lives in the
// file-scope array below instead of a caller workspace.
//
// The array is CROSS_NTT_NOALLOC_SCRATCH_BYTES (16 MiB) per GPU and is held
// by every GPU that loads this library until the process exits.  The
// intermediate takes two words per input word (ntt_tmp_words), so one call
// converts at most CROSS_NTT_NOALLOC_MAX_WORDS = 2 Mi input words.  Its device
// address is looked up once per device and cached for the process, so
// cudaDeviceReset after the first call is not supported.  All calls
// share it and it keeps the previous call's contents (the NTT overwrites
// every word it reads, so nothing needs clearing); calls that overlap on the
// GPU -- on different streams, or from different host threads -- race on it,
// so issue them on one stream.
#include <mutex>

#include "internal.hpp"

namespace {

constexpr size_t kScratchWords = CROSS_NTT_NOALLOC_SCRATCH_BYTES / sizeof(uint32_t);

static __device__ __align__(256) uint32_t g_ntt_noalloc_scratch[kScratchWords];

constexpr int kMaxDevices = 256;
std::mutex g_scratch_mu;
uint32_t* g_scratch_addr[kMaxDevices] = {};

// Device address of g_ntt_noalloc_scratch on the current device.  In host
// code the array's name is only a stand-in, so the address is looked up once
// per device, with that device current, and cached.
int scratch_on_current_device(uint32_t** out) {
  int dev = -1;
  CROSS_CHECK_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) {
    cross::set_error("cross_ntt_noalloc: device ordinal %d out of range", dev);
    return CROSS_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    CROSS_CHECK_CUDA(cudaGetSymbolAddress(&p, g_ntt_noalloc_scratch));
    g_scratch_addr[dev] = (uint32_t*)p;
  }
  *out = g_scratch_addr[dev];
  return CROSS_OK;
}

}  // namespace

extern "C" int cross_ntt_noalloc(cross_ntt_plan P, int inverse, const uint32_t* in, uint32_t* out, int64_t batch,
                                 void* stream) {
  CROSS_REQUIRE(P && batch >= 0 && (batch == 0 || (in && out)), "cross_ntt_noalloc: null argument or negative batch");
  if (batch == 0) return CROSS_OK;
  const int64_t N = (int64_t)P->r * P->c;
  const int M = P->M;
  const int64_t words = cross::ntt_tmp_words(P, batch * M);
  if (words > (int64_t)kScratchWords) {
    cross::set_error(
        "cross_ntt_noalloc: batch %lld x %d limbs x N %lld needs %lld scratch words, which exceeds the %zu-word "
        "(%u MiB) static scratch; use cross_ntt with a workspace",
        (long long)batch, M, (long long)N, (long long)words, kScratchWords, CROSS_NTT_NOALLOC_SCRATCH_BYTES >> 20);
    return CROSS_ERR_WORKSPACE;
  }
  uint32_t* scratch = nullptr;
  int rc = scratch_on_current_device(&scratch);
  if (rc) return rc;
  return cross::ntt_run(P, inverse != 0, cross::LP{in, M * N, N}, cross::LPo{out, M * N, N}, batch, M, P->identity,
                        scratch, (cudaStream_t)stream);
}
