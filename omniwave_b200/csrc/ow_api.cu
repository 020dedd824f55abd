// C-ABI entry points of libomniwave_b200.so (declared in
// include/omniwave_b200.h).  This layer validates arguments, derives the
// problem shape, carves the caller's workspace and picks the kernel family:
// the tensor-core path for bf16/f16 compute on the shapes it covers, the
// CUDA-core path otherwise.  There is no host fallback: every call either
// launches device work or returns an error code.

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "ow_common.cuh"
#include "ow_internal.h"

namespace ow {

static thread_local char g_err[1024] = {0};
static std::atomic<uint64_t> g_launches{0};

void count_launches(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

// Process-wide (autograd runs backward calls on its own device threads).
static std::atomic<void*> g_prof[4][2] = {};

void profile_mark(int kernel, bool after, cudaStream_t st) {
  void* e = g_prof[kernel][after ? 1 : 0].load(std::memory_order_acquire);
  if (e) cudaEventRecord((cudaEvent_t)e, st);
}

// The device fault word: one int in every device's copy of this library's
// device memory.  Kernels of every file receive its address as an argument,
// so a bounded wait that gives up anywhere is reported in this one place.
static __device__ int g_fault_word = 0;
constexpr int kMaxDevices = 64;
static std::mutex g_fault_mu;
static int* g_fault_ptr[kMaxDevices] = {};
static std::atomic<uint32_t> g_probe_ns{0};

int fault_word(int** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_error("fault word: no usable current device (%s)", cudaGetErrorString(e));
    return OW_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lk(g_fault_mu);
  if (!g_fault_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_fault_word);
    if (e != cudaSuccess || !p) {
      set_error("fault word: cudaGetSymbolAddress failed on device %d: %s", dev, cudaGetErrorString(e));
      return OW_ERR_CUDA;
    }
    g_fault_ptr[dev] = (int*)p;
  }
  *out = g_fault_ptr[dev];
  return OW_OK;
}

uint32_t wait_probe_ns() { return g_probe_ns.load(std::memory_order_relaxed); }

int device_sm_count() {
  static std::atomic<int> cached[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  int n = cached[dev].load(std::memory_order_relaxed);
  if (n <= 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = 148;
    }
    cached[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

void clear_error() { g_err[0] = 0; }

static bool valid_dtype(int dt) {
  return dt == OW_DTYPE_F32 || dt == OW_DTYPE_F64 || dt == OW_DTYPE_BF16 || dt == OW_DTYPE_F16;
}

// Shape checks shared by every entry point.
static int make_prob(const ow_bigemm_args_t* a, Prob* p, bool need_ptrs) {
  OW_CHECK_ARG(a != nullptr, "args is NULL");
  const ow_route_t& r = a->route;
  OW_CHECK_ARG(r.batch > 0 && r.height > 0 && r.width > 0 && r.channels > 0,
               "batch/height/width/channels must be positive (got %d,%d,%d,%d)", r.batch,
               r.height, r.width, r.channels);
  OW_CHECK_ARG(r.g == 16, "spatial tile g must be 16 (got %d)", r.g);
  OW_CHECK_ARG(r.d > 0 && r.rd > 0, "channel tile d and rd must be positive (got %d,%d)", r.d, r.rd);
  const int64_t n = (int64_t)r.height * r.width;
  OW_CHECK_ARG(n < (1LL << 30), "too many tokens (%lld)", (long long)n);
  OW_CHECK_ARG(r.q_s == (int)((n + r.g - 1) / r.g), "q_s=%d does not match ceil(H*W/g)=%lld",
               r.q_s, (long long)((n + r.g - 1) / r.g));
  OW_CHECK_ARG(r.q_c == (r.channels + r.d - 1) / r.d, "q_c=%d does not match ceil(C/d)=%d", r.q_c,
               (r.channels + r.d - 1) / r.d);
  OW_CHECK_ARG(valid_dtype(a->x_dtype) && valid_dtype(a->w_dtype) && valid_dtype(a->compute_dtype),
               "invalid dtype code (x=%d w=%d compute=%d)", a->x_dtype, a->w_dtype, a->compute_dtype);
  OW_CHECK_ARG(r.ch_stride >= 0, "ch_stride hint must be >= 0 (got %d)", r.ch_stride);
  const int64_t tiles = (int64_t)r.batch * r.q_s;
  OW_CHECK_ARG(tiles < (1LL << 31) - 1 && r.q_c < 65535, "grid too large (B*q_s=%lld, q_c=%d)",
               (long long)tiles, r.q_c);
  if (need_ptrs) {
    OW_CHECK_ARG(r.tok_idx && r.ch_idx, "route tables are NULL");
    OW_CHECK_ARG(a->x && a->a_u && a->a_v && a->a_o && a->b_u && a->b_v && a->b_o && a->gamma,
                 "an input pointer is NULL");
    OW_CHECK_ARG(!a->rstd || a->norm_w, "block mode (rstd != NULL) needs norm_w");
  }
  p->B = r.batch; p->H = r.height; p->W = r.width; p->C = r.channels; p->N = (int)n;
  p->Qs = r.q_s; p->Qc = r.q_c; p->g = r.g; p->d = r.d; p->rd = r.rd;
  p->tok = r.tok_idx; p->ch = r.ch_idx;
  p->chs = r.ch_stride;
  return OW_OK;
}

static bool use_tc(const ow_bigemm_args_t* a, const Prob& p) {
  const char* why = nullptr;
  return (a->compute_dtype == OW_DTYPE_BF16 || a->compute_dtype == OW_DTYPE_F16) &&
         tc_supported(a, p, &why);
}

static size_t measure(const ow_bigemm_args_t* a, const Prob& p, bool bwd) {
  Carver c(nullptr);
  ow_bigemm_grads_t dummy{};
  if (use_tc(a, p)) {
    if (bwd) tc_backward(a, &dummy, p, nullptr, c);
    else tc_forward(a, p, nullptr, c);
  } else {
    if (bwd) simt_backward(a, &dummy, p, nullptr, c);
    else simt_forward(a, p, nullptr, c);
  }
  return c.used + 256;
}

// Entry points of other translation units reuse the same validation,
// dispatch and workspace sizing.
int api_make_prob(const ow_bigemm_args_t* a, Prob* p) { return make_prob(a, p, true); }
bool api_use_tc(const ow_bigemm_args_t* a, const Prob& p) { return use_tc(a, p); }
size_t api_measure(const ow_bigemm_args_t* a, const Prob& p, bool bwd) { return measure(a, p, bwd); }

}  // namespace ow

using namespace ow;

extern "C" {

int ow_abi_version(void) { return OW_ABI_VERSION; }

uint64_t ow_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int ow_profile_events(int kernel, void* start, void* stop) {
  if (kernel < OW_PROF_FWD || kernel > OW_PROF_FPACK) {
    set_error("ow_profile_events: unknown kernel %d", kernel);
    return OW_ERR_INVALID;
  }
  g_prof[kernel][0].store(start, std::memory_order_release);
  g_prof[kernel][1].store(stop, std::memory_order_release);
  return OW_OK;
}

const char* ow_last_error(void) { return g_err; }

int ow_device_supported(int device) {
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
  return (major == 10 && minor == 0) ? 1 : 0;
}

int ow_device_fault(int device, int reset) {
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) return -1;
  if (cudaSetDevice(device) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  int v = -1;
  if (cudaDeviceSynchronize() == cudaSuccess &&
      cudaMemcpyFromSymbol(&v, g_fault_word, sizeof(int)) == cudaSuccess) {
    if (reset && v != 0) {
      const int z = 0;
      if (cudaMemcpyToSymbol(g_fault_word, &z, sizeof(int)) != cudaSuccess) v = -1;
    }
  } else {
    v = -1;
  }
  cudaSetDevice(prev);
  return v;
}

int ow_debug_wait_probe(uint32_t probe_ns) {
  if (probe_ns > 1000000000u) {
    set_error("ow_debug_wait_probe: %u ns is longer than the 1 s limit of the self-check", probe_ns);
    return OW_ERR_INVALID;
  }
  g_probe_ns.store(probe_ns, std::memory_order_relaxed);
  return OW_OK;
}

size_t ow_bigemm_workspace_size(const ow_bigemm_args_t* args, int for_backward) {
  Prob p;
  if (make_prob(args, &p, false) != OW_OK) return 0;
  return measure(args, p, for_backward != 0);
}

int ow_rmsnorm_rstd(const void* x, int32_t x_dtype, int32_t compute_dtype, int64_t rows,
                    int32_t channels, double eps, void* rstd, void* stream) {
  clear_error();
  OW_CHECK_ARG(x && rstd, "x or rstd is NULL");
  OW_CHECK_ARG(rows > 0 && channels > 0, "rows and channels must be positive");
  return rmsnorm_rstd(x, x_dtype, compute_dtype, rows, channels, eps, rstd, stream);
}

int ow_bigemm_fwd(const ow_bigemm_args_t* args, void* stream) {
  clear_error();
  Prob p;
  OW_RETURN_IF(make_prob(args, &p, true));
  OW_CHECK_ARG(args->out, "out is NULL");
  OW_CHECK_ARG(valid_dtype(args->out_dtype), "invalid out dtype %d", args->out_dtype);
  const size_t need = measure(args, p, false);
  if (!args->workspace || args->workspace_bytes < need) {
    set_error("forward needs %zu workspace bytes, got %zu", need, args->workspace_bytes);
    return OW_ERR_WORKSPACE;
  }
  Carver ws(args->workspace);
  if (use_tc(args, p)) return tc_forward(args, p, stream, ws);
  return simt_forward(args, p, stream, ws);
}

int ow_bigemm_bwd(const ow_bigemm_args_t* args, const ow_bigemm_grads_t* grads, void* stream) {
  clear_error();
  Prob p;
  OW_RETURN_IF(make_prob(args, &p, true));
  OW_CHECK_ARG(grads && grads->dout && grads->dx && grads->da_u && grads->da_v && grads->da_o &&
                   grads->db_u && grads->db_v && grads->db_o && grads->dgamma,
               "a gradient pointer is NULL");
  OW_CHECK_ARG(!args->rstd || grads->dnorm_w, "block mode needs dnorm_w");
  OW_CHECK_ARG(valid_dtype(args->out_dtype), "invalid out dtype %d", args->out_dtype);
  const size_t need = measure(args, p, true);
  if (!args->workspace || args->workspace_bytes < need) {
    set_error("backward needs %zu workspace bytes, got %zu", need, args->workspace_bytes);
    return OW_ERR_WORKSPACE;
  }
  Carver ws(args->workspace);
  if (use_tc(args, p)) return tc_backward(args, grads, p, stream, ws);
  return simt_backward(args, grads, p, stream, ws);
}

}  // extern "C"
