// Allocation-free forward entry point: ow_bigemm_fwd_noalloc.
//
// Some callers cannot allocate device memory at the point where they run
// BiGEMM: plugin hosts that hand a kernel only its input and output buffers,
// code inside a region where the process's allocator must not be entered, or
// runtimes that forbid cudaMalloc after start-up.  For them this entry point
// takes its scratch from a fixed-size array that lives in the library's own
// device memory (a file-scope __device__ array, present on every GPU that
// loads the library until the process exits) instead of a caller workspace.
//
// Contract:
//  - Scratch is at most kNoAllocScratchBytes; a call whose shapes need more is
//    rejected with OW_ERR_WORKSPACE before anything is launched.
//  - The device address of the array is looked up once per device, with that
//    device current, on the first call made while it is current; that first
//    call should come before any stream capture.
//  - Nothing in the scratch has to start at zero: the forward's preparation
//    kernel writes every byte the main kernel reads.
//  - Every call shares the one array and it keeps the last call's contents,
//    so calls whose executions overlap on the GPU (different streams, or
//    concurrent host threads) race on it.  Serialise them.
//  - It allocates nothing: no cudaMalloc, no cudaFree, no allocating library
//    routine.

#include <mutex>

#include "ow_common.cuh"
#include "ow_internal.h"

namespace ow {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;  // 4 MiB
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device.  In host code
// the array's name is only a host-side stand-in, so the address must come
// from cudaGetSymbolAddress with the device current.
int scratch_on_current_device(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_error("ow_bigemm_fwd_noalloc: cudaGetDevice failed: %s", cudaGetErrorString(e));
    return OW_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("ow_bigemm_fwd_noalloc: device index %d out of range", dev);
    return OW_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_error("ow_bigemm_fwd_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                cudaGetErrorString(e));
      return OW_ERR_CUDA;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return OW_OK;
}

}  // namespace
}  // namespace ow

using namespace ow;

extern "C" {

size_t ow_noalloc_scratch_limit(void) { return kNoAllocScratchBytes; }

int ow_bigemm_fwd_noalloc(const ow_bigemm_args_t* args, void* stream) {
  clear_error();
  Prob p;
  OW_RETURN_IF(api_make_prob(args, &p));
  OW_CHECK_ARG(args->out, "out is NULL");
  OW_CHECK_ARG(args->out_dtype == OW_DTYPE_F32 || args->out_dtype == OW_DTYPE_F64 ||
                   args->out_dtype == OW_DTYPE_BF16 || args->out_dtype == OW_DTYPE_F16,
               "invalid out dtype %d", args->out_dtype);
  const size_t need = api_measure(args, p, false);
  if (need > kNoAllocScratchBytes) {
    set_error("ow_bigemm_fwd_noalloc: these shapes need %zu bytes of scratch, more than its fixed %zu-byte "
              "limit; use ow_bigemm_fwd with a caller workspace",
              need, kNoAllocScratchBytes);
    return OW_ERR_WORKSPACE;
  }
  void* scratch = nullptr;
  OW_RETURN_IF(scratch_on_current_device(&scratch));
  Carver ws(scratch);
  if (api_use_tc(args, p)) return tc_forward(args, p, stream, ws);
  return simt_forward(args, p, stream, ws);
}

}  // extern "C"
