// decode_static.cu -- pa_paged_attention_v3_noalloc: the split-KV decode with
// its scratch memory held inside the library, so the caller allocates nothing.
//
// Who needs this: hosts that hand the library only the pointers they already
// own and have no way (or no permission) to get more device memory at call
// time -- an FFI host with no device allocator of its own (a plain C program or
// a language runtime that receives device buffers from elsewhere), or a serving
// loop whose device memory is reserved up front in a fixed arena, where an
// allocation in the middle of a decode step could fail or wait on the
// allocator.  The regular entry points take a caller-provided workspace; this
// one takes none.
//
// How: the scratch (plan tables, merge counters, split partials) lives in the
// file-scope array g_noalloc_scratch below, PA_NOALLOC_SCRATCH_BYTES (8 MiB) per
// device, held by every GPU that loads the library until the process exits.
// Host code cannot pass the array's name to a kernel (on the host it is only a
// stand-in, not a device address), so on the first call on each device -- with
// that device current -- the library asks the runtime for the array's device
// address with cudaGetSymbolAddress and caches it.  That first call on a device
// should therefore come before any stream capture.  The cached address belongs
// to the device's context of that moment: cudaDeviceReset destroys it, so the
// entry point must not be used across a reset of the device in the same
// process.  Every call on a device shares the one array and leaves its
// contents behind.  Nothing from one call reaches the next: the merge counters
// and the abort flag carry a tag of the launch that wrote them (a new tag per
// launch), so values left by an earlier call read as zero, and the plan tables
// are rebuilt by every call (in shared memory for up to 1024 sequences, by the
// plan kernel into the array above that).  Two calls whose work overlaps on
// the GPU (different streams, or different host threads) race on the array,
// so callers must order them.  Requests that need more scratch than the array
// holds are rejected with PA_ERR_TOO_LARGE before anything is launched.
#include <mutex>
#include <utility>
#include <vector>

#include "common.cuh"
#include "decode_host.h"

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[PA_NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch on the current device (looked up once per
// device).
int noalloc_scratch(void** out) {
  static std::mutex mu;
  static std::vector<std::pair<int, void*>> addr;  // (device, address)
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return pa::cuda_status(e);
  std::lock_guard<std::mutex> lk(mu);
  for (const auto& a : addr)
    if (a.first == dev) {
      *out = a.second;
      return PA_OK;
    }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || p == nullptr) return pa::cuda_status(e != cudaSuccess ? e : cudaErrorInvalidSymbol);
  addr.push_back({dev, p});
  *out = p;
  return PA_OK;
}

}  // namespace

extern "C" int pa_paged_attention_v3_noalloc(
    float* out, float* lse, const float* q, const void* k_cache, const void* v_cache,
    int kv_dtype, const int32_t* block_tables, const int32_t* context_lens, int64_t num_seqs,
    int64_t num_heads, int64_t num_kv_heads, int64_t head_dim, int64_t block_size,
    int64_t num_blocks, int64_t max_blocks, double scale, int64_t num_splits,
    int32_t* dev_status, void* stream) {
  pa::decode::DecodeArgs a;
  a.out = out;
  a.lse = lse;
  a.q = q;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.dtype = kv_dtype;
  a.block_tables = block_tables;
  a.context_lens = context_lens;
  a.B = num_seqs;
  a.H = num_heads;
  a.HKV = num_kv_heads;
  a.D = head_dim;
  a.BS = block_size;
  a.NB = num_blocks;
  a.MB = max_blocks;
  a.scale = scale;
  a.num_splits = num_splits;
  a.dev_status = dev_status;
  a.qlen = 1;
  a.empty_fill = __builtin_nanf("");  // NaN rows for empty sequences, as the v3 entry point
  // size check first: nothing is touched or launched for an oversized request
  size_t need = 0;
  int st = pa::decode::workspace_bytes(a, &need);
  if (st) return st;
  if (need > (size_t)PA_NOALLOC_SCRATCH_BYTES) return PA_ERR_TOO_LARGE;
  if (num_seqs == 0) return PA_OK;
  void* scratch = nullptr;
  st = noalloc_scratch(&scratch);
  if (st) return st;
  return pa::decode::launch(a, scratch, (size_t)PA_NOALLOC_SCRATCH_BYTES,
                            static_cast<cudaStream_t>(stream));
}
