// Internal interfaces between the C-ABI layer (ow_api.cu) and the kernel
// files.  Not part of the public ABI.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include "omniwave_b200.h"

namespace ow {

// Shape of one call, derived and validated from ow_route_t.
struct Prob {
  int B, H, W, C, N;
  int Qs, Qc, g, d, rd;
  const int32_t* tok;  // [Qs*g]
  const int32_t* ch;   // [Qc*d]
  int chs;             // channel-layout hint of the route (ow_route_t.ch_stride)
#ifdef __CUDACC__
  __host__ __device__
#endif
  int64_t BQ() const { return (int64_t)B * Qs; }
#ifdef __CUDACC__
  __host__ __device__
#endif
  int64_t ntiles() const { return BQ() * Qc; }
};

#ifdef __CUDACC__
// Channel layout of group qc, one int per group (``layout[qc]``):
//   0            generic: channels gathered one by one through the table;
//   S + 16 * c0  the group's channels are c0, c0 + S, ..., c0 + S (D - 1)
//                with S in {1, 2, 4, 8} and C % 8 == 0, where
//                S == 1: one aligned run (c0 % 8 == 0, c0 + D <= C), so
//                        16-byte vector accesses apply directly;
//                S > 1:  c0 < S and S D <= C, so every 64-channel half of
//                        the group lies in the aligned span [64 S h, 64 S (h+1))
//                        of the row, read with 16-byte vectors and
//                        de-interleaved (the stride-Q_c groups of radix
//                        routes at levels 1 and 2, routing.py:107-121).
// One warp per group, called by every thread of the grid.
__host__ __device__ constexpr int layout_stride(int v) { return v & 15; }
__host__ __device__ constexpr int layout_c0(int v) { return v >> 4; }

template <int D>
__device__ __forceinline__ void contig_flags(const Prob& p, int* layout) {
  const int lane = threadIdx.x & 31;
  const int gw = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int nw = (int)((gridDim.x * blockDim.x) >> 5);
  for (int qc = gw; qc < p.Qc; qc += nw) {
    const int c0 = p.ch[qc * D];
    const int S = D > 1 ? p.ch[qc * D + 1] - c0 : 1;
    bool ok = S == 1 || S == 2 || S == 4 || S == 8;
    for (int k = lane; k < D && ok; k += 32) ok &= p.ch[qc * D + k] == c0 + S * k;
    ok = __all_sync(0xffffffffu, ok) && (p.C % 8 == 0);
    if (S == 1) ok = ok && (c0 % 8 == 0) && (c0 + D <= p.C);
    else ok = ok && (c0 < S) && (S * D <= p.C);
    if (lane == 0) layout[qc] = ok ? S + 16 * c0 : 0;
  }
}
#endif

// Workspace carve-up helper: hands out aligned sub-ranges of one buffer and
// tracks the total size (a dry run with base == nullptr measures it).
struct Carver {
  char* base;
  size_t used = 0;
  explicit Carver(void* b) : base((char*)b) {}
  void* take(size_t bytes) {
    used = (used + 255) / 256 * 256;
    void* p = base ? base + used : nullptr;
    used += bytes;
    return p;
  }
};

// Validation / dispatch / workspace sizing shared by every entry point.
int api_make_prob(const ow_bigemm_args_t* a, Prob* p);
bool api_use_tc(const ow_bigemm_args_t* a, const Prob& p);
size_t api_measure(const ow_bigemm_args_t* a, const Prob& p, bool bwd);

// CUDA-core path (exact fp32 / fp64; also any shape the tensor path lacks).
int simt_forward(const ow_bigemm_args_t* a, const Prob& p, void* stream, Carver& ws);
int simt_backward(const ow_bigemm_args_t* a, const ow_bigemm_grads_t* gr, const Prob& p,
                  void* stream, Carver& ws);
int rmsnorm_rstd(const void* x, int x_dtype, int compute_dtype, int64_t rows, int C,
                 double eps, void* rstd, void* stream);

// Tensor-core path (bf16/f16 compute, g=16, d in {64,128}, rd=2d).
bool tc_supported(const ow_bigemm_args_t* a, const Prob& p, const char** why);
// Forward with TMA row gathers and tensor-core token mixes (ow_tcf.cu): true
// when it covers this call (contiguous channel groups, 16-bit x, operator
// or block mode); tcf_forward() then runs it with the weight images the forward prep
// kernel wrote (``img``, ``amat``, ``gg``, ``nwc``, ``layout``).
bool tcf_covers(const ow_bigemm_args_t* a, const Prob& p);
int tcf_forward(const ow_bigemm_args_t* a, const Prob& p, const unsigned char* img, const uint16_t* amat,
                const float* gg, const float* nwc, const int* layout, void* stream);
int tc_forward(const ow_bigemm_args_t* a, const Prob& p, void* stream, Carver& ws);
// The forward's pre-pass: [P_u | P_v] operand images per item (ow_tc_bwd.cu).
int tc_pack_forward(const ow_bigemm_args_t* a, const Prob& p, const uint16_t* amat, const float* nwc,
                    const int* contig, unsigned char* packed, void* stream);

// The library's device fault word on the current device (one int per device,
// shared by every kernel file; kernels get its address as an argument).
// The first call on a device looks the address up.
int fault_word(int** out);
// Wait-timeout self-check setting (ow_debug_wait_probe); 0 when off.
uint32_t wait_probe_ns();
// Streaming multiprocessors of the current device (cached per device).
int device_sm_count();
// cuTensorMapEncodeTiled for a 16-bit tensor of ``rank`` dimensions (dims and
// byte strides of dimensions 1.. innermost first), 128-byte swizzle, zero
// fill out of range; ``map`` points at a CUtensorMap.  ``who`` prefixes the
// error message.
int encode_tiled_map(void* map, bool bf16, int rank, const void* base, const uint64_t* dims,
                     const uint64_t* strides, const uint32_t* box, const char* who);

// RMSNorm backward of block mode from the gradient w.r.t. the normalised
// input (``dxn``, f32 or the 16-bit compute type; CUDA cores, row-wise).  norm_bwd_take() carves its partials from
// the workspace (also in a dry run); norm_bwd_run() launches it.
struct NormBwd {
  float* part;
  int grid, nwarps;  // blocks of the norm backward; partial rows it leaves for the column sum
};
NormBwd norm_bwd_take(int64_t rows, int C, Carver& ws);
int norm_bwd_run(const NormBwd& nb, const void* x, int x_dt, const void* dout, int dout_dt, const float* rstd,
                 const float* nw, const void* dxn, int dxn_dt, int64_t rows, int C, void* dx, void* dnorm_w, int w_dt,
                 void* stream);
int tc_backward(const ow_bigemm_args_t* a, const ow_bigemm_grads_t* gr, const Prob& p,
                void* stream, Carver& ws);

}  // namespace ow
