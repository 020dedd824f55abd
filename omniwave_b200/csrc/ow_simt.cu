// CUDA-core (SIMT) BiGEMM path: exact fp32 / fp64 arithmetic for any tile
// shape.  It is the precision anchor of the library (the reference's fp32
// tolerance of 1e-4 relative cannot be met with bf16 operands) and serves
// shapes the tensor-core path does not cover.
//
// Forward: one CTA per (spatial tile, channel group).  The tile is gathered
// through the route tables straight from the NHWC input (reference
// pack_tiles, omniweave/ops/reference.py:16-64), the three contractions and
// the silu gate run out of shared memory (reference.py:147-171) and the
// result is stored straight to its NHWC position (unpack_tiles :67-117).
//
// Backward: the same per-tile CTA recomputes the forward, walks the chain
// rule back to the input gradient and leaves the per-tile operands of the
// weight gradients in the workspace; a deterministic split reduction then
// forms dA_* (summed over all tiles) and dB_* (summed per channel group).

#include <algorithm>
#include <cstdarg>
#include <type_traits>

#include "ow_common.cuh"
#include "ow_internal.h"

namespace ow {

namespace {

constexpr int kThreads = 256;

// Offsets (in compute elements) of the weight copies the prep step writes.
struct WOff {
  int64_t au, av, ao, bu, bv, bo, gg, nw, total;
  WOff(const Prob& p) {
    int64_t gg2 = (int64_t)p.g * p.g, bsz = (int64_t)p.Qc * p.d * p.rd;
    au = 0; av = gg2; ao = 2 * gg2; bu = 3 * gg2; bv = bu + bsz; bo = bv + bsz;
    gg = bo + bsz; nw = gg + (int64_t)p.Qc * p.d; total = nw + p.C;
  }
};

// ---------------------------------------------------------------------------
// Weight preparation: copy (and round through the compute dtype) into the
// compute type; build the grouped LayerScale gamma[ch_idx] * ch_mask
// (reference.py:168-170).
// ---------------------------------------------------------------------------
template <typename TW, typename TC>
__global__ void prep_convert_kernel(const TW* __restrict__ src, TC* __restrict__ dst, int64_t n,
                                    int round_dt) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = round_through(load_as<TC>(src, i), round_dt);
}

template <typename TW, typename TC>
__global__ void prep_gamma_kernel(const TW* __restrict__ gamma, const int32_t* __restrict__ ch,
                                  int64_t n, int C, TC* __restrict__ gg) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    int c = ch[i];
    gg[i] = (c < C) ? load_as<TC>(gamma, c) : TC(0);
  }
}

// One element of a gathered tile (optionally RMS-normalised).  The rounding
// steps follow the reference block (block.py:83-85) and the autocast cast of
// the einsum operands to the compute dtype.
template <typename TX, typename TC>
__device__ __forceinline__ TC tile_elem(const Prob& p, const TX* __restrict__ x,
                                        const TC* __restrict__ rstd, const TC* __restrict__ nw,
                                        int x_dt, int c_dt, int b, int tok, int ch) {
  if (tok >= p.N || ch >= p.C) return TC(0);
  int64_t row = (int64_t)b * p.N + tok;
  TC v = load_as<TC>(x, row * p.C + ch);
  if (rstd) {
    v = round_through(v * rstd[row], x_dt);
    v = round_through(v * nw[ch], x_dt);
  }
  return round_through(v, c_dt);
}

// ---------------------------------------------------------------------------
// Forward tile kernel.
// ---------------------------------------------------------------------------
template <typename TX, typename TO, typename TC>
__global__ void __launch_bounds__(kThreads)
simt_fwd_kernel(Prob p, const TX* __restrict__ x, const TC* __restrict__ rstd,
                const TC* __restrict__ wts, WOff wo, int x_dt, int c_dt,
                const float* __restrict__ scale, int residual, TO* __restrict__ out) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int g = p.g, d = p.d, rd = p.rd;
  TC* sA = reinterpret_cast<TC*>(smem_raw);
  TC* sT = sA + 3 * g * g;
  TC* sPu = sT + g * d;
  TC* sPv = sPu + g * d;
  TC* sY = sPv + g * d;
  TC* sZ = sY + g * d;
  const int bq = blockIdx.x, qc = blockIdx.y;
  const int b = bq / p.Qs, qs = bq - b * p.Qs;
  const TC* nw = rstd ? wts + wo.nw : nullptr;
  const TC* Bu = wts + wo.bu + (int64_t)qc * d * rd;
  const TC* Bv = wts + wo.bv + (int64_t)qc * d * rd;
  const TC* Bo = wts + wo.bo + (int64_t)qc * rd * d;
  const TC* gg = wts + wo.gg + (int64_t)qc * d;

  for (int i = threadIdx.x; i < 3 * g * g; i += blockDim.x) sA[i] = wts[wo.au + i];
  for (int idx = threadIdx.x; idx < g * d; idx += blockDim.x) {
    int i = idx / d, k = idx - i * d;
    sT[idx] = tile_elem<TX, TC>(p, x, rstd, nw, x_dt, c_dt, b, p.tok[qs * g + i], p.ch[qc * d + k]);
  }
  __syncthreads();
  // Token mix: P = A T.
  for (int idx = threadIdx.x; idx < g * d; idx += blockDim.x) {
    int i = idx / d, k = idx - i * d;
    TC pu = 0, pv = 0;
    for (int j = 0; j < g; ++j) {
      TC t = sT[j * d + k];
      pu += sA[i * g + j] * t;
      pv += sA[g * g + i * g + j] * t;
    }
    sPu[idx] = round_through(pu, c_dt);
    sPv[idx] = round_through(pv, c_dt);
  }
  __syncthreads();
  // Channel mix and gate: Z = silu(P_u B_u) * (P_v B_v).
  for (int idx = threadIdx.x; idx < g * rd; idx += blockDim.x) {
    int i = idx / rd, e = idx - i * rd;
    TC u = 0, v = 0;
    for (int k = 0; k < d; ++k) {
      u += sPu[i * d + k] * Bu[(int64_t)k * rd + e];
      v += sPv[i * d + k] * Bv[(int64_t)k * rd + e];
    }
    u = round_through(u, c_dt);
    v = round_through(v, c_dt);
    TC s = round_through(u * ow_sigmoid(u), c_dt);
    sZ[idx] = round_through(s * v, c_dt);
  }
  __syncthreads();
  // Output projection Y = Z B_o.
  for (int idx = threadIdx.x; idx < g * d; idx += blockDim.x) {
    int i = idx / d, k = idx - i * d;
    TC y = 0;
    for (int e = 0; e < rd; ++e) y += sZ[i * rd + e] * Bo[(int64_t)e * d + k];
    sY[idx] = round_through(y, c_dt);
  }
  __syncthreads();
  // delta = A_o Y, masked, scaled by gamma (and drop-path), scattered.
  const TC sb = scale ? TC(scale[b]) : TC(1);
  for (int idx = threadIdx.x; idx < g * d; idx += blockDim.x) {
    int i = idx / d, k = idx - i * d;
    int tok = p.tok[qs * g + i], ch = p.ch[qc * d + k];
    if (tok >= p.N || ch >= p.C) continue;
    TC du = 0;
    for (int j = 0; j < g; ++j) du += sA[2 * g * g + i * g + j] * sY[j * d + k];
    du = round_through(du, c_dt);
    TC delta = du * gg[k] * sb;
    int64_t off = ((int64_t)b * p.N + tok) * p.C + ch;
    if (residual) delta += load_as<TC>(x, off);
    out[off] = Elem<TO>::from(delta);
  }
}

// ---------------------------------------------------------------------------
// Backward tile kernel.  Intermediates live in the workspace (global memory,
// block-local, ordered by __syncthreads).
// ---------------------------------------------------------------------------
template <typename TC>
struct Scratch {
  TC *T, *Pu, *Pv, *Y, *G, *dY, *dPu, *dPv;  // [ntiles][g][d]
  TC *U, *V, *Z, *dU, *dV;                   // [ntiles][g][rd]
  TC* dgg;                                   // [ntiles][d]
};

template <typename TX, typename TO, typename TC>
__global__ void __launch_bounds__(kThreads)
simt_bwd_tile_kernel(Prob p, const TX* __restrict__ x, const TC* __restrict__ rstd,
                     const TC* __restrict__ wts, WOff wo, int x_dt, int c_dt,
                     const float* __restrict__ scale, const TO* __restrict__ dout,
                     TC* __restrict__ dxn, TX* __restrict__ dx, Scratch<TC> s) {
  __shared__ TC sA[3 * 16 * 16];
  const int g = p.g, d = p.d, rd = p.rd;
  const int bq = blockIdx.x, qc = blockIdx.y;
  const int b = bq / p.Qs, qs = bq - b * p.Qs;
  const int64_t t = (int64_t)qc * p.BQ() + bq;
  const TC* nw = rstd ? wts + wo.nw : nullptr;
  const TC* Bu = wts + wo.bu + (int64_t)qc * d * rd;
  const TC* Bv = wts + wo.bv + (int64_t)qc * d * rd;
  const TC* Bo = wts + wo.bo + (int64_t)qc * rd * d;
  const TC* gg = wts + wo.gg + (int64_t)qc * d;
  TC *T = s.T + t * g * d, *Pu = s.Pu + t * g * d, *Pv = s.Pv + t * g * d, *Y = s.Y + t * g * d;
  TC *G = s.G + t * g * d, *dY = s.dY + t * g * d, *dPu = s.dPu + t * g * d, *dPv = s.dPv + t * g * d;
  TC *U = s.U + t * g * rd, *V = s.V + t * g * rd, *Z = s.Z + t * g * rd;
  TC *dU = s.dU + t * g * rd, *dV = s.dV + t * g * rd;
  const TC* Au = sA;
  const TC* Av = sA + g * g;
  const TC* Ao = sA + 2 * g * g;

  for (int i = threadIdx.x; i < 3 * g * g; i += blockDim.x) sA[i] = wts[wo.au + i];
  for (int idx = threadIdx.x; idx < g * d; idx += blockDim.x) {
    int i = idx / d, k = idx - i * d;
    T[idx] = tile_elem<TX, TC>(p, x, rstd, nw, x_dt, c_dt, b, p.tok[qs * g + i], p.ch[qc * d + k]);
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < g * d; idx += blockDim.x) {
    int i = idx / d, k = idx - i * d;
    TC pu = 0, pv = 0;
    for (int j = 0; j < g; ++j) {
      TC tv = T[j * d + k];
      pu += Au[i * g + j] * tv;
      pv += Av[i * g + j] * tv;
    }
    Pu[idx] = round_through(pu, c_dt);
    Pv[idx] = round_through(pv, c_dt);
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < g * rd; idx += blockDim.x) {
    int i = idx / rd, e = idx - i * rd;
    TC u = 0, v = 0;
    for (int k = 0; k < d; ++k) {
      u += Pu[i * d + k] * Bu[(int64_t)k * rd + e];
      v += Pv[i * d + k] * Bv[(int64_t)k * rd + e];
    }
    u = round_through(u, c_dt);
    v = round_through(v, c_dt);
    U[idx] = u;
    V[idx] = v;
    TC sl = round_through(u * ow_sigmoid(u), c_dt);
    Z[idx] = round_through(sl * v, c_dt);
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < g * d; idx += blockDim.x) {
    int i = idx / d, k = idx - i * d;
    TC y = 0;
    for (int e = 0; e < rd; ++e) y += Z[i * rd + e] * Bo[(int64_t)e * d + k];
    Y[idx] = round_through(y, c_dt);
  }
  __syncthreads();
  // Gathered upstream gradient G' (mask, drop-path scale), G = G' * gamma, and
  // the per-tile LayerScale gradient sum_i G'[i,k] * (A_o Y)[i,k].
  const TC sb = scale ? TC(scale[b]) : TC(1);
  for (int k = threadIdx.x; k < d; k += blockDim.x) {
    int ch = p.ch[qc * d + k];
    TC acc = 0;
    for (int i = 0; i < g; ++i) {
      int tok = p.tok[qs * g + i];
      TC gp = 0;
      if (tok < p.N && ch < p.C)
        gp = load_as<TC>(dout, ((int64_t)b * p.N + tok) * p.C + ch) * sb;
      TC du = 0;
      for (int j = 0; j < g; ++j) du += Ao[i * g + j] * Y[j * d + k];
      acc += gp * round_through(du, c_dt);
      G[i * d + k] = gp * gg[k];
    }
    s.dgg[t * d + k] = acc;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < g * d; idx += blockDim.x) {
    int i = idx / d, k = idx - i * d;
    TC a = 0;
    for (int j = 0; j < g; ++j) a += Ao[j * g + i] * G[j * d + k];
    dY[idx] = a;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < g * rd; idx += blockDim.x) {
    int i = idx / rd, e = idx - i * rd;
    TC dz = 0;
    for (int k = 0; k < d; ++k) dz += dY[i * d + k] * Bo[(int64_t)e * d + k];
    TC u = U[idx], v = V[idx];
    TC sg = ow_sigmoid(u);
    dU[idx] = dz * v * sg * (TC(1) + u * (TC(1) - sg));
    dV[idx] = dz * u * sg;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < g * d; idx += blockDim.x) {
    int i = idx / d, k = idx - i * d;
    TC a = 0, c = 0;
    for (int e = 0; e < rd; ++e) {
      a += dU[i * rd + e] * Bu[(int64_t)k * rd + e];
      c += dV[i * rd + e] * Bv[(int64_t)k * rd + e];
    }
    dPu[idx] = a;
    dPv[idx] = c;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < g * d; idx += blockDim.x) {
    int i = idx / d, k = idx - i * d;
    int tok = p.tok[qs * g + i], ch = p.ch[qc * d + k];
    if (tok >= p.N || ch >= p.C) continue;
    TC a = 0;
    for (int j = 0; j < g; ++j) a += Au[j * g + i] * dPu[j * d + k] + Av[j * g + i] * dPv[j * d + k];
    int64_t off = ((int64_t)b * p.N + tok) * p.C + ch;
    if (dxn) dxn[off] = a;
    else dx[off] = Elem<TX>::from(a);
  }
}

// ---------------------------------------------------------------------------
// Deterministic split reduction:
//   part[z][m][n] = sum_{t in split z} sum_r L[t*lt + r*lr + m*lm] * R[t*rt + r*rr + n*rn]
// batched over ``nb`` independent problems (channel groups).
// ---------------------------------------------------------------------------
template <typename TC>
struct RedSpec {
  const TC* L; int64_t lt, lr, lm, lb;
  const TC* R; int64_t rt, rr, rn, rb;
  int64_t NT; int NR, M, N, S, nb;
  TC* part;  // [nb][S][M][N]
};

template <typename TC>
__global__ void __launch_bounds__(256) simt_reduce_kernel(RedSpec<TC> s) {
  const int n = blockIdx.x * 16 + threadIdx.x;
  const int m = blockIdx.y * 16 + threadIdx.y;
  const int z = blockIdx.z % s.S, bi = blockIdx.z / s.S;
  if (m >= s.M || n >= s.N) return;
  const int64_t t0 = s.NT * z / s.S, t1 = s.NT * (z + 1) / s.S;
  const TC* L = s.L + bi * s.lb + m * s.lm;
  const TC* R = s.R + bi * s.rb + n * s.rn;
  TC acc = 0;
  for (int64_t t = t0; t < t1; ++t)
    for (int r = 0; r < s.NR; ++r) acc += L[t * s.lt + r * s.lr] * R[t * s.rt + r * s.rr];
  s.part[(((int64_t)bi * s.S + z) * s.M + m) * s.N + n] = acc;
}

// out[bi][m][n] = sum_z part[bi][z][m][n]  (cast to the gradient dtype)
template <typename TC, typename TW>
__global__ void simt_sum_parts_kernel(const TC* __restrict__ part, int S, int64_t MN, int nb,
                                      TW* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < MN * nb;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t bi = i / MN, mn = i - bi * MN;
    TC acc = 0;
    for (int z = 0; z < S; ++z) acc += part[(bi * S + z) * MN + mn];
    out[i] = Elem<TW>::from(acc);
  }
}

// out[c] = sum_z part[z][c] for c < C: per-warp partials of the RMSNorm
// weight gradient, S of them.  One 1024-thread block per 32 columns: warp w
// sums rows w, w + 32, w + 64, ... in that order (eight loads in flight),
// then warp 0 adds the 32 warp sums in order, so the result is bitwise
// reproducible while 32 x ceil(C / 32) warps share the rows.
template <typename TC, typename TW>
__global__ void __launch_bounds__(1024) simt_col_sum_kernel(const TC* __restrict__ part, int S, int C,
                                                            TW* __restrict__ out) {
  __shared__ TC red[32][33];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lane;
  const int cc = c < C ? c : C - 1;  // clamped column: loads stay in bounds, result unused
  TC acc = 0;
  for (int z0 = w; z0 < S; z0 += 32 * 8) {
    TC v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int z = z0 + 32 * k;
      v[k] = part[(int64_t)(z < S ? z : S - 1) * C + cc];
    }
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (z0 + 32 * k < S) acc += v[k];
  }
  red[w][lane] = acc;
  __syncthreads();
  if (w == 0) {
    TC t = 0;
    for (int k = 0; k < 32; ++k) t += red[k][lane];
    if (c < C) out[c] = Elem<TW>::from(t);
  }
}

template <typename TC>
int launch_col_sum(const TC* part, int S, int C, void* out, int w_dt, cudaStream_t st) {
  const int g = (C + 31) / 32;
  switch (w_dt) {
    case OW_DTYPE_F32: launch(simt_col_sum_kernel<TC, float>, g, 1024, 0, st, part, S, C, (float*)out); break;
    case OW_DTYPE_F64: launch(simt_col_sum_kernel<TC, double>, g, 1024, 0, st, part, S, C, (double*)out); break;
    case OW_DTYPE_BF16: launch(simt_col_sum_kernel<TC, __nv_bfloat16>, g, 1024, 0, st, part, S, C, (__nv_bfloat16*)out); break;
    case OW_DTYPE_F16: launch(simt_col_sum_kernel<TC, __half>, g, 1024, 0, st, part, S, C, (__half*)out); break;
    default: set_error("unsupported weight dtype"); return OW_ERR_UNSUPPORTED;
  }
  OW_CHECK_LAUNCH("norm weight reduction");
  return OW_OK;
}

// dgamma[ch[q,k]] = sum over tiles of channel group q of dgg[t][k].
template <typename TC, typename TW>
__global__ void simt_dgamma_kernel(const TC* __restrict__ dgg, int64_t BQ, int Qc, int d,
                                   const int32_t* __restrict__ ch, int C, TW* __restrict__ dgamma) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= Qc * d) return;
  int q = i / d, k = i - q * d;
  int c = ch[i];
  if (c >= C) return;
  TC acc = 0;
  const TC* src = dgg + (int64_t)q * BQ * d + k;
  for (int64_t t = 0; t < BQ; ++t) acc += src[t * d];
  dgamma[c] = Elem<TW>::from(acc);
}

// ---------------------------------------------------------------------------
// RMSNorm statistics and backward (block mode).
// ---------------------------------------------------------------------------
template <typename TX, typename TC>
__global__ void rstd_kernel(const TX* __restrict__ x, int64_t rows, int C, double eps, int x_dt,
                            TC* __restrict__ rstd, int vec) {
  const int lane = threadIdx.x & 31;
  int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  constexpr int EV = 16 / (int)sizeof(TX);  // elements per 16-byte vector
  for (; row < rows; row += nwarps) {
    const TX* xr = x + row * C;
    double acc = 0;
    if (vec) {  // 16-byte loads (C % EV == 0, row starts aligned)
      for (int c = lane * EV; c < C; c += 32 * EV) {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(xr + c));
        const TX* e = reinterpret_cast<const TX*>(&u);
#pragma unroll
        for (int k = 0; k < EV; ++k) {
          const float v = Elem<TX>::to_f(e[k]);
          acc += (double)(v * v);
        }
      }
    } else {
      for (int c = lane; c < C; c += 32) {
        float v = Elem<TX>::to_f(xr[c]);
        acc += (double)(v * v);
      }
    }
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    // mean in float32 (x.float().square().mean), cast to x's dtype, + eps, rsqrt
    float var32 = (float)(acc / C);
    TC v = round_through((TC)var32, x_dt);
    v = round_through(v + (TC)eps, x_dt);
    TC r = round_through(TC(1) / sqrt(v), x_dt);
    if (lane == 0) rstd[row] = r;
  }
}

// Vectorised statistics: a row is ``lpr`` lanes (16 or 32) of 16-byte loads,
// a warp covers 32 / lpr rows per step and RU steps per iteration, and every
// lane issues all of its RU loads before it reduces any of them, so each lane
// keeps RU loads in flight (one row per warp left rows of 256 B with a single
// load per lane and the kernel latency-bound).  Same finishing steps as
// rstd_kernel; each 16-byte vector's squares are summed in f32 (at most eight
// terms), the rest in double.
template <typename TX, typename TC>
__device__ __forceinline__ double sumsq16(const uint4& u) {
  const TX* e = reinterpret_cast<const TX*>(&u);
  if constexpr (sizeof(TX) == 8) {
    double a = 0;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const double v = (double)e[k];
      a += v * v;
    }
    return a;
  } else {
    // The vector's (at most eight) squares in f32, then double from there on.
    float a = 0.f;
#pragma unroll
    for (int k = 0; k < 16 / (int)sizeof(TX); ++k) {
      const float v = Elem<TX>::to_f(e[k]);
      a = fmaf(v, v, a);
    }
    return (double)a;
  }
}

template <typename TX, typename TC>
__global__ void __launch_bounds__(256) rstd_vec_kernel(const TX* __restrict__ x, int64_t rows, int C, double eps,
                                                       int x_dt, TC* __restrict__ rstd, int lpr) {
  constexpr int RU = 4;
  constexpr int EV = 16 / (int)sizeof(TX);
  const int lane = threadIdx.x & 31;
  const int rpw = 32 / lpr, sub = lane / lpr, sl = lane % lpr;
  const int vpr = C / EV;  // 16-byte vectors per row
  const int64_t gw = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r0 = gw * rpw * RU; r0 < rows; r0 += nwarps * rpw * RU) {
    double acc[RU];
#pragma unroll
    for (int u = 0; u < RU; ++u) acc[u] = 0;
    for (int v0 = sl; v0 < vpr; v0 += lpr) {
      uint4 q[RU];
#pragma unroll
      for (int u = 0; u < RU; ++u) {
        const int64_t row = r0 + u * rpw + sub;
        // Rows past the end load row 0 (always valid); their sums are dropped.
        q[u] = __ldg(reinterpret_cast<const uint4*>(x + (row < rows ? row : 0) * C) + v0);
      }
#pragma unroll
      for (int u = 0; u < RU; ++u) acc[u] += sumsq16<TX, TC>(q[u]);
    }
#pragma unroll
    for (int u = 0; u < RU; ++u) {
      for (int o = lpr >> 1; o > 0; o >>= 1) acc[u] += __shfl_xor_sync(0xffffffffu, acc[u], o);
      const int64_t row = r0 + u * rpw + sub;
      if (sl == 0 && row < rows) {
        float var32 = (float)(acc[u] / C);
        TC v = round_through((TC)var32, x_dt);
        v = round_through(v + (TC)eps, x_dt);
        rstd[row] = round_through(TC(1) / sqrt(v), x_dt);
      }
    }
  }
}

// One warp per row; lane l owns channels l, l+32, ... (J per lane, C <= 32*J).
// The norm-weight gradient is accumulated per warp; when the block's eight
// warp sums fit 32 KB of shared memory they are added in warp order and the
// block writes one partial row (COMBINE), else each warp writes its own.  The
// partial rows are then summed in a fixed order (simt_col_sum_kernel), so the
// result is bitwise reproducible.
template <typename TC, int J>
constexpr bool norm_combine() { return 8 * 32 * J * sizeof(TC) <= 32768; }

template <typename TX, typename TO, typename TC, typename TD, int J>
__global__ void __launch_bounds__(256)
norm_bwd_kernel(const TX* __restrict__ x, const TC* __restrict__ rstd, const TC* __restrict__ nw,
                const TD* __restrict__ dxn, const TO* __restrict__ dout, int64_t rows, int C,
                TX* __restrict__ dx, TC* __restrict__ dw_part) {
  constexpr bool COMBINE = norm_combine<TC, J>();
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int64_t gw = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  TC acc[J];
#pragma unroll
  for (int j = 0; j < J; ++j) acc[j] = 0;
  for (int64_t row = gw; row < rows; row += nwarps) {
    const int64_t base = row * C;
    const TC r = rstd[row];
    TC xv[J], gn[J], dv[J];
    TC inner = 0;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      int c = lane + 32 * j;
      xv[j] = c < C ? load_as<TC>(x, base + c) : TC(0);
      gn[j] = c < C ? load_as<TC>(dxn, base + c) : TC(0);
      dv[j] = c < C ? load_as<TC>(dout, base + c) : TC(0);  // requested before the reduction
      inner += c < C ? gn[j] * nw[c] * xv[j] : TC(0);
    }
    for (int o = 16; o > 0; o >>= 1) inner += __shfl_xor_sync(0xffffffffu, inner, o);
    const TC coef = r * r * r * inner / TC(C);
#pragma unroll
    for (int j = 0; j < J; ++j) {
      int c = lane + 32 * j;
      if (c < C) {
        TC v = dv[j] + r * nw[c] * gn[j] - xv[j] * coef;
        dx[base + c] = Elem<TX>::from(v);
        acc[j] += gn[j] * xv[j] * r;
      }
    }
  }
  if constexpr (COMBINE) {
    __shared__ TC red[8][32 * J];
#pragma unroll
    for (int j = 0; j < J; ++j) red[wib][lane + 32 * j] = acc[j];
    __syncthreads();
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
      TC t = 0;
#pragma unroll
      for (int k = 0; k < 8; ++k) t += red[k][c];
      dw_part[(int64_t)blockIdx.x * C + c] = t;
    }
  } else {
#pragma unroll
    for (int j = 0; j < J; ++j) {
      int c = lane + 32 * j;
      if (c < C) dw_part[gw * C + c] = acc[j];
    }
  }
}

// Number of partial rows launch_norm_bwd leaves for the column sum.
template <typename TC>
int norm_parts(int grid, int C) {
  bool comb;
  if (C <= 128) comb = norm_combine<TC, 4>();
  else if (C <= 256) comb = norm_combine<TC, 8>();
  else if (C <= 512) comb = norm_combine<TC, 16>();
  else if (C <= 1024) comb = norm_combine<TC, 32>();
  else comb = norm_combine<TC, 64>();
  return comb ? grid : grid * 8;
}

// Blocks of the norm backward: one warp per row, enough blocks to fill the
// GPU several times over, while the partials (8 warps x C per block) stay
// under 16 MB.
inline int norm_grid_for(int64_t rows, int C) {
  const int64_t cap = std::max<int64_t>(296, std::min<int64_t>(1184, (int64_t)(1 << 19) / C));
  return (int)std::max<int64_t>(1, std::min<int64_t>((rows + 63) / 64, cap));
}

template <typename TX, typename TO, typename TC, typename TD>
int launch_norm_bwd(int grid, cudaStream_t st, const TX* x, const TC* rstd, const TC* nw,
                    const TD* dxn, const TO* dout, int64_t rows, int C, TX* dx, TC* dw_part) {
  if (C <= 128) launch(norm_bwd_kernel<TX, TO, TC, TD, 4>, grid, 256, 0, st, x, rstd, nw, dxn, dout, rows, C, dx, dw_part);
  else if (C <= 256) launch(norm_bwd_kernel<TX, TO, TC, TD, 8>, grid, 256, 0, st, x, rstd, nw, dxn, dout, rows, C, dx, dw_part);
  else if (C <= 512) launch(norm_bwd_kernel<TX, TO, TC, TD, 16>, grid, 256, 0, st, x, rstd, nw, dxn, dout, rows, C, dx, dw_part);
  else if (C <= 1024) launch(norm_bwd_kernel<TX, TO, TC, TD, 32>, grid, 256, 0, st, x, rstd, nw, dxn, dout, rows, C, dx, dw_part);
  else if (C <= 2048) launch(norm_bwd_kernel<TX, TO, TC, TD, 64>, grid, 256, 0, st, x, rstd, nw, dxn, dout, rows, C, dx, dw_part);
  else {
    set_error("block mode supports at most 2048 channels (got %d)", C);
    return OW_ERR_UNSUPPORTED;
  }
  OW_CHECK_LAUNCH("norm_bwd_kernel");
  return OW_OK;
}

inline int grid_for(int64_t n, int threads = 256, int cap = 148 * 16) {
  int64_t b = (n + threads - 1) / threads;
  return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

// Launch the weight preparation into ``w`` (compute type TC).
template <typename TC, typename TW>
int prep_weights_t(const ow_bigemm_args_t* a, const Prob& p, const WOff& wo, TC* w,
                   cudaStream_t st) {
  const int rdt = a->compute_dtype;
  auto conv = [&](const void* src, int64_t off, int64_t n, int round_dt) {
    launch(prep_convert_kernel<TW, TC>, grid_for(n), 256, 0, st, (const TW*)src, w + off, n, round_dt);
  };
  int64_t gg2 = (int64_t)p.g * p.g, bsz = (int64_t)p.Qc * p.d * p.rd;
  conv(a->a_u, wo.au, gg2, rdt);
  conv(a->a_v, wo.av, gg2, rdt);
  conv(a->a_o, wo.ao, gg2, rdt);
  conv(a->b_u, wo.bu, bsz, rdt);
  conv(a->b_v, wo.bv, bsz, rdt);
  conv(a->b_o, wo.bo, bsz, rdt);
  int64_t ng = (int64_t)p.Qc * p.d;
  launch(prep_gamma_kernel<TW, TC>, grid_for(ng), 256, 0, st, (const TW*)a->gamma, p.ch, ng, p.C, w + wo.gg);
  if (a->rstd) conv(a->norm_w, wo.nw, p.C, OW_DTYPE_F64);  // no rounding
  OW_CHECK_LAUNCH("prep_weights");
  return OW_OK;
}

template <typename TC>
int prep_weights(const ow_bigemm_args_t* a, const Prob& p, const WOff& wo, TC* w, cudaStream_t st) {
  switch (a->w_dtype) {
    case OW_DTYPE_F32: return prep_weights_t<TC, float>(a, p, wo, w, st);
    case OW_DTYPE_F64: return prep_weights_t<TC, double>(a, p, wo, w, st);
    case OW_DTYPE_BF16: return prep_weights_t<TC, __nv_bfloat16>(a, p, wo, w, st);
    case OW_DTYPE_F16: return prep_weights_t<TC, __half>(a, p, wo, w, st);
  }
  set_error("unsupported weight dtype %d", a->w_dtype);
  return OW_ERR_UNSUPPORTED;
}

// dtype dispatch over (x, out) storage types for a given compute type.
template <typename TC, typename F>
int dispatch_io(int x_dt, int o_dt, F&& f) {
#define OW_CASE_O(TX)                                                          \
  switch (o_dt) {                                                              \
    case OW_DTYPE_F32: return f((TX*)nullptr, (float*)nullptr);                \
    case OW_DTYPE_BF16: return f((TX*)nullptr, (__nv_bfloat16*)nullptr);       \
    case OW_DTYPE_F16: return f((TX*)nullptr, (__half*)nullptr);               \
    default: break;                                                            \
  }
  if constexpr (sizeof(TC) == 8) {
    if (x_dt == OW_DTYPE_F64 && o_dt == OW_DTYPE_F64) return f((double*)nullptr, (double*)nullptr);
  } else {
    switch (x_dt) {
      case OW_DTYPE_F32: OW_CASE_O(float) break;
      case OW_DTYPE_BF16: OW_CASE_O(__nv_bfloat16) break;
      case OW_DTYPE_F16: OW_CASE_O(__half) break;
      default: break;
    }
  }
#undef OW_CASE_O
  set_error("unsupported dtype combination x=%s out=%s for compute %s", dtype_name(x_dt),
            dtype_name(o_dt), sizeof(TC) == 8 ? "float64" : "float32");
  return OW_ERR_UNSUPPORTED;
}

template <typename TC>
int simt_forward_t(const ow_bigemm_args_t* a, const Prob& p, cudaStream_t st, Carver& ws) {
  WOff wo(p);
  TC* w = (TC*)ws.take(wo.total * sizeof(TC));
  if (!ws.base) return OW_OK;
  OW_RETURN_IF(prep_weights<TC>(a, p, wo, w, st));
  size_t smem = sizeof(TC) * (3 * p.g * p.g + 4 * p.g * p.d + p.g * p.rd);
  return dispatch_io<TC>(a->x_dtype, a->out_dtype, [&](auto* tx, auto* to) -> int {
    using TX = std::remove_pointer_t<decltype(tx)>;
    using TO = std::remove_pointer_t<decltype(to)>;
    auto kern = simt_fwd_kernel<TX, TO, TC>;
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) {
        set_error("simt forward: shared memory %zu bytes not available: %s", smem, cudaGetErrorString(e));
        return OW_ERR_UNSUPPORTED;
      }
    }
    dim3 grid((unsigned)p.BQ(), (unsigned)p.Qc);
    launch(kern, grid, kThreads, smem, st, p, (const TX*)a->x, (const TC*)a->rstd, w, wo, a->x_dtype,
                                        a->compute_dtype, a->sample_scale, a->residual, (TO*)a->out);
    OW_CHECK_LAUNCH("simt_fwd_kernel");
    return OW_OK;
  });
}

template <typename TC>
int reduce_launch(const RedSpec<TC>& base, TC* part, void* out, int w_dt, cudaStream_t st) {
  RedSpec<TC> s = base;
  s.part = part;
  dim3 grid((s.N + 15) / 16, (s.M + 15) / 16, s.S * s.nb);
  launch(simt_reduce_kernel<TC>, grid, dim3(16, 16), 0, st, s);
  int64_t MN = (int64_t)s.M * s.N;
  int gsz = grid_for(MN * s.nb);
  switch (w_dt) {
    case OW_DTYPE_F32: launch(simt_sum_parts_kernel<TC, float>, gsz, 256, 0, st, part, s.S, MN, s.nb, (float*)out); break;
    case OW_DTYPE_F64: launch(simt_sum_parts_kernel<TC, double>, gsz, 256, 0, st, part, s.S, MN, s.nb, (double*)out); break;
    case OW_DTYPE_BF16: launch(simt_sum_parts_kernel<TC, __nv_bfloat16>, gsz, 256, 0, st, part, s.S, MN, s.nb, (__nv_bfloat16*)out); break;
    case OW_DTYPE_F16: launch(simt_sum_parts_kernel<TC, __half>, gsz, 256, 0, st, part, s.S, MN, s.nb, (__half*)out); break;
  }
  OW_CHECK_LAUNCH("simt_reduce");
  return OW_OK;
}

inline int splits_for(int64_t NT, int M, int N, int nb) {
  int64_t blocks = (int64_t)((N + 15) / 16) * ((M + 15) / 16) * nb;
  int64_t want = (148 * 8 + blocks - 1) / blocks;
  if (want > NT) want = NT;
  if (want < 1) want = 1;
  if (want > 1024) want = 1024;
  return (int)want;
}

template <typename TC>
int simt_backward_t(const ow_bigemm_args_t* a, const ow_bigemm_grads_t* gr, const Prob& p,
                    cudaStream_t st, Carver& ws) {
  WOff wo(p);
  const int64_t nt = p.ntiles(), gd = (int64_t)p.g * p.d, grd = (int64_t)p.g * p.rd;
  TC* w = (TC*)ws.take(wo.total * sizeof(TC));
  Scratch<TC> s;
  TC** small[] = {&s.T, &s.Pu, &s.Pv, &s.Y, &s.G, &s.dY, &s.dPu, &s.dPv};
  for (TC** q : small) *q = (TC*)ws.take(nt * gd * sizeof(TC));
  TC** big[] = {&s.U, &s.V, &s.Z, &s.dU, &s.dV};
  for (TC** q : big) *q = (TC*)ws.take(nt * grd * sizeof(TC));
  s.dgg = (TC*)ws.take(nt * p.d * sizeof(TC));
  const int64_t rows = (int64_t)p.B * p.N;
  const bool block = a->rstd != nullptr;
  TC* dxn = block ? (TC*)ws.take(rows * p.C * sizeof(TC)) : nullptr;

  // Reduction specs (partials carved after the fixed buffers).
  const int g = p.g, d = p.d, rd = p.rd;
  const int64_t BQ = p.BQ();
  RedSpec<TC> rs[6];
  void* outs[6] = {gr->da_u, gr->da_v, gr->da_o, gr->db_u, gr->db_v, gr->db_o};
  // dA_u = sum_t dPu_t T_t^T ; dA_v ; dA_o = sum_t G_t Y_t^T
  auto tokspec = [&](const TC* L, const TC* R) {
    RedSpec<TC> r{};
    r.L = L; r.lt = gd; r.lr = 1; r.lm = d; r.lb = 0;
    r.R = R; r.rt = gd; r.rr = 1; r.rn = d; r.rb = 0;
    r.NT = nt; r.NR = d; r.M = g; r.N = g; r.nb = 1;
    r.S = splits_for(nt, g, g, 1);
    return r;
  };
  // dB = sum over tiles of one channel group of L_t^T R_t.
  auto chspec = [&](const TC* L, int kl, const TC* R, int kr) {
    RedSpec<TC> r{};
    r.L = L; r.lt = (int64_t)g * kl; r.lr = kl; r.lm = 1; r.lb = BQ * g * kl;
    r.R = R; r.rt = (int64_t)g * kr; r.rr = kr; r.rn = 1; r.rb = BQ * g * kr;
    r.NT = BQ; r.NR = g; r.M = kl; r.N = kr; r.nb = p.Qc;
    r.S = splits_for(BQ, kl, kr, p.Qc);
    return r;
  };
  rs[0] = tokspec(s.dPu, s.T);
  rs[1] = tokspec(s.dPv, s.T);
  rs[2] = tokspec(s.G, s.Y);
  rs[3] = chspec(s.Pu, d, s.dU, rd);
  rs[4] = chspec(s.Pv, d, s.dV, rd);
  rs[5] = chspec(s.Z, rd, s.dY, d);
  TC* parts[6];
  for (int i = 0; i < 6; ++i)
    parts[i] = (TC*)ws.take((size_t)rs[i].nb * rs[i].S * rs[i].M * rs[i].N * sizeof(TC));
  int nw_warps = 0;
  TC* dw_part = nullptr;
  int norm_grid = 0;
  if (block) {
    norm_grid = norm_grid_for(rows, p.C);
    nw_warps = norm_parts<TC>(norm_grid, p.C);
    dw_part = (TC*)ws.take((size_t)norm_grid * 8 * p.C * sizeof(TC));
  }
  if (!ws.base) return OW_OK;

  OW_RETURN_IF(prep_weights<TC>(a, p, wo, w, st));
  int rc = dispatch_io<TC>(a->x_dtype, a->out_dtype, [&](auto* tx, auto* to) -> int {
    using TX = std::remove_pointer_t<decltype(tx)>;
    using TO = std::remove_pointer_t<decltype(to)>;
    dim3 grid((unsigned)BQ, (unsigned)p.Qc);
    launch(simt_bwd_tile_kernel<TX, TO, TC>, grid, kThreads, 0, st, 
        p, (const TX*)a->x, (const TC*)a->rstd, w, wo, a->x_dtype, a->compute_dtype,
        a->sample_scale, (const TO*)gr->dout, dxn, block ? nullptr : (TX*)gr->dx, s);
    OW_CHECK_LAUNCH("simt_bwd_tile_kernel");
    if (block)
      return launch_norm_bwd<TX, TO, TC, TC>(norm_grid, st, (const TX*)a->x, (const TC*)a->rstd,
                                         w + wo.nw, dxn, (const TO*)gr->dout, rows, p.C,
                                         (TX*)gr->dx, dw_part);
    return OW_OK;
  });
  OW_RETURN_IF(rc);
  for (int i = 0; i < 6; ++i) OW_RETURN_IF(reduce_launch<TC>(rs[i], parts[i], outs[i], a->w_dtype, st));
  int gsz = (p.Qc * p.d + 127) / 128;
  switch (a->w_dtype) {
    case OW_DTYPE_F32: launch(simt_dgamma_kernel<TC, float>, gsz, 128, 0, st, s.dgg, BQ, p.Qc, d, p.ch, p.C, (float*)gr->dgamma); break;
    case OW_DTYPE_F64: launch(simt_dgamma_kernel<TC, double>, gsz, 128, 0, st, s.dgg, BQ, p.Qc, d, p.ch, p.C, (double*)gr->dgamma); break;
    case OW_DTYPE_BF16: launch(simt_dgamma_kernel<TC, __nv_bfloat16>, gsz, 128, 0, st, s.dgg, BQ, p.Qc, d, p.ch, p.C, (__nv_bfloat16*)gr->dgamma); break;
    case OW_DTYPE_F16: launch(simt_dgamma_kernel<TC, __half>, gsz, 128, 0, st, s.dgg, BQ, p.Qc, d, p.ch, p.C, (__half*)gr->dgamma); break;
  }
  OW_CHECK_LAUNCH("simt_dgamma_kernel");
  if (block) return launch_col_sum<TC>(dw_part, nw_warps, p.C, gr->dnorm_w, a->w_dtype, st);
  return OW_OK;
}

}  // namespace

int simt_forward(const ow_bigemm_args_t* a, const Prob& p, void* stream, Carver& ws) {
  cudaStream_t st = (cudaStream_t)stream;
  if (a->compute_dtype == OW_DTYPE_F64) return simt_forward_t<double>(a, p, st, ws);
  return simt_forward_t<float>(a, p, st, ws);
}

int simt_backward(const ow_bigemm_args_t* a, const ow_bigemm_grads_t* gr, const Prob& p,
                  void* stream, Carver& ws) {
  cudaStream_t st = (cudaStream_t)stream;
  if (a->compute_dtype == OW_DTYPE_F64) return simt_backward_t<double>(a, gr, p, st, ws);
  return simt_backward_t<float>(a, gr, p, st, ws);
}

NormBwd norm_bwd_take(int64_t rows, int C, Carver& ws) {
  NormBwd nb;
  nb.grid = norm_grid_for(rows, C);
  nb.nwarps = norm_parts<float>(nb.grid, C);
  nb.part = (float*)ws.take((size_t)nb.grid * 8 * C * sizeof(float));
  return nb;
}

int norm_bwd_run(const NormBwd& nb, const void* x, int x_dt, const void* dout, int dout_dt, const float* rstd,
                 const float* nw, const void* dxn, int dxn_dt, int64_t rows, int C, void* dx, void* dnorm_w,
                 int w_dt, void* stream) {
  cudaStream_t st = (cudaStream_t)stream;
  auto run = [&](auto* tx, auto* to) -> int {
    using TX = std::remove_pointer_t<decltype(tx)>;
    using TO = std::remove_pointer_t<decltype(to)>;
    switch (dxn_dt) {
      case OW_DTYPE_F32:
        return launch_norm_bwd<TX, TO, float, float>(nb.grid, st, (const TX*)x, rstd, nw, (const float*)dxn,
                                                     (const TO*)dout, rows, C, (TX*)dx, nb.part);
      case OW_DTYPE_BF16:
        return launch_norm_bwd<TX, TO, float, __nv_bfloat16>(nb.grid, st, (const TX*)x, rstd, nw,
                                                             (const __nv_bfloat16*)dxn, (const TO*)dout, rows, C,
                                                             (TX*)dx, nb.part);
      case OW_DTYPE_F16:
        return launch_norm_bwd<TX, TO, float, __half>(nb.grid, st, (const TX*)x, rstd, nw, (const __half*)dxn,
                                                      (const TO*)dout, rows, C, (TX*)dx, nb.part);
      default:
        set_error("norm backward: unsupported gradient dtype %s", dtype_name(dxn_dt));
        return OW_ERR_UNSUPPORTED;
    }
  };
  int rc = dispatch_io<float>(x_dt, dout_dt, run);
  OW_RETURN_IF(rc);
  return launch_col_sum<float>(nb.part, nb.nwarps, C, dnorm_w, w_dt, st);
}

int rmsnorm_rstd(const void* x, int x_dtype, int compute_dtype, int64_t rows, int C, double eps,
                 void* rstd, void* stream) {
  cudaStream_t st = (cudaStream_t)stream;
  const int es = (int)dtype_size(x_dtype);
  const int vec = ((uintptr_t)x % 16 == 0) && (C * es % 16 == 0);
  // Vectorised path: 16 lanes per row when a row is at most 16 vectors and
  // that divides evenly, else 32.
  const int vpr = vec ? C * es / 16 : 0;
  const int lpr = vpr > 0 && vpr <= 16 && 16 % vpr == 0 ? 16 : 32;
  const int64_t rows_per_block = 8LL * (32 / lpr) * 4;  // 8 warps x rows per step x 4 steps
  const int vgrid = (int)std::max<int64_t>(1, std::min<int64_t>((rows + rows_per_block - 1) / rows_per_block,
                                                                 (int64_t)device_sm_count() * 16));
  int grid = grid_for(rows * 32, 256, 148 * 16);
  if (compute_dtype == OW_DTYPE_F64) {
    if (x_dtype != OW_DTYPE_F64) {
      set_error("rmsnorm: float64 compute needs float64 input");
      return OW_ERR_UNSUPPORTED;
    }
    if (vec) launch(rstd_vec_kernel<double, double>, vgrid, 256, 0, st, (const double*)x, rows, C, eps, x_dtype, (double*)rstd, lpr);
    else launch(rstd_kernel<double, double>, grid, 256, 0, st, (const double*)x, rows, C, eps, x_dtype, (double*)rstd, vec);
  } else {
    auto go = [&](auto* tx) {
      using TX = std::remove_pointer_t<decltype(tx)>;
      if (vec) launch(rstd_vec_kernel<TX, float>, vgrid, 256, 0, st, (const TX*)x, rows, C, eps, x_dtype, (float*)rstd, lpr);
      else launch(rstd_kernel<TX, float>, grid, 256, 0, st, (const TX*)x, rows, C, eps, x_dtype, (float*)rstd, vec);
    };
    switch (x_dtype) {
      case OW_DTYPE_F32: go((float*)nullptr); break;
      case OW_DTYPE_BF16: go((__nv_bfloat16*)nullptr); break;
      case OW_DTYPE_F16: go((__half*)nullptr); break;
      default:
        set_error("rmsnorm: unsupported input dtype %s", dtype_name(x_dtype));
        return OW_ERR_UNSUPPORTED;
    }
  }
  OW_CHECK_LAUNCH("rstd_kernel");
  return OW_OK;
}

}  // namespace ow
