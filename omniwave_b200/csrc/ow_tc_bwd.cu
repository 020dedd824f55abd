// Tensor-core BiGEMM backward for sm_100a (bf16 / f16 compute, g = 16,
// d in {64, 128}, rd = 2d).
//
// The gradient of the forward (reference.py:147-171, taken by autograd in the
// reference) is, per tile with G' = mask * scale * dOut and G = G' * gamma:
//
//   H   = A_o^T G'            dZ = (H * gamma) B_o^T  (Z = silu(U) * V)
//   dU  = dZ * V * silu'(U)   dV = dZ * silu(U)
//   dP_u = dU B_u^T           dP_v = dV B_v^T
//   dT  = A_u^T dP_u + A_v^T dP_v                          -> dX (scattered)
//   dA_u = sum dP_u T^T,  dA_v = sum dP_v T^T,  dA_o = sum G (Z B_o)^T
//   dB_u = sum P_u^T dU,  dB_v = sum P_v^T dV
//   M_o  = sum (A_o Z)^T G' = sum Z^T H  ->  dB_o = M_o * gamma,  dgamma = sum_e B_o * M_o
//
// gamma is folded into the B_o^T weight stages (dZ = H (B_o diag(gamma))^T),
// so H serves both dZ and M_o and no token mix of Z is needed.
//
// The weight gradients sum over every tile of a channel group; their f32
// accumulators (3 x d x rd) do not fit one SM's 512 TMEM columns next to the
// working set at d = 128, so the work runs as three CTA roles:
//
//   DGRAD  (any item)      U, V, dZ -> dU, dV -> dP_u, dP_v (TMEM)   -> dX, dA_u, dA_v
//   UV(h)  (one group)     U, V, dZ on rd half h -> dU, dV -> TMEM += dU^T P_u, dV^T P_v
//   O      (one group)     U, V -> Z; TMEM Y += Z B_o, M_o += Z^T H  -> dA_o
//
// Every role needs the same per-item operands (P_u, P_v, H, G', T).  A
// pack kernel with many CTAs per SM gathers x and dOut through the route
// tables once per item and writes those five operands as pre-swizzled
// images; the persistent role kernel then streams them (and the weight
// chunk images) into shared memory with bulk copies issued by one producer
// warp, so its compute warps only run the per-chunk elementwise work and the
// per-item epilogue while the tensor work of the next item proceeds.
//
// The UV and O weight-gradient products read the token-major tiles already
// in shared memory through MN-major UMMA descriptors; the DGRAD epilogue
// reads dP straight out of TMEM in the mma.sync fragment layout
// (tcgen05.ld 16x256b) for the 16x16 token-mix gradients.  Each CTA writes
// f32 partials; a reduction kernel sums them in a fixed order (bitwise
// reproducible).  Per-role thread layout: 8 compute warps, one MMA-issuing
// warp that owns TMEM, one producer warp issuing the bulk copies.

#include <algorithm>
#include <array>
#include <map>
#include <mutex>
#include <cmath>
#include <type_traits>

#include "ow_common.cuh"
#include "ow_internal.h"
#include "ow_sm100.cuh"

namespace ow {
namespace {

using namespace sm100;

constexpr int BM = 128;
constexpr int NCOMP_WARPS = 8;
constexpr int NCOMP = NCOMP_WARPS * 32;
constexpr int MMA_WARP = NCOMP_WARPS;
constexpr int PROD_WARP = NCOMP_WARPS + 1;
constexpr int TC_THREADS = (NCOMP_WARPS + 2) * 32;
constexpr int STG_LD = 72;
constexpr int STG_BYTES = BM * STG_LD * 2;
constexpr int TMEM_COLS = 512;

enum Role { R_DGRAD = 0, R_UV = 1, R_O = 2 };

template <int D>
struct BCfg {
  static constexpr int RD = 2 * D;
  static constexpr int NH = RD / 128;           // 128-feature halves
  // Pipeline step: SC features per sub-chunk.  The U/V/dZ accumulators of two
  // sub-chunks are live in TMEM at once (one being read by the compute warps
  // while the tensor pipe fills the other), which at d = 128 leaves room for
  // 32 features per sub-chunk next to the d x 2d f32 accumulators.
  static constexpr int SC = D == 64 ? 64 : 32;
  static constexpr int NSUB = RD / SC;          // sub-chunks per item (DGRAD, O)
  static constexpr int NSUB_UV = 128 / SC;      // sub-chunks per UV half
  static constexpr int SPC = 64 / SC;           // sub-chunks per 64-feature chunk
  static constexpr int P_BYTES = BM * D * 2;
  static constexpr int Z_BYTES = BM * 64 * 2;   // one 64-column SW128 atom of 128 rows (16 KB)
  // Weight images per channel group: for every sub-chunk s one contiguous
  // stage [B_u | B_v | B_o^T] of SC features x D channels (K-major, SC rows),
  // then for every 64-feature chunk k the slice B_o[k] as D rows x 64 features.
  static constexpr int SUB_BYTES = SC * D * 2;
  static constexpr int A_BYTES = 3 * SUB_BYTES;
  static constexpr int BO_BYTES = D * 64 * 2;
  static constexpr int QC_IMG = NSUB * A_BYTES + (RD / 64) * BO_BYTES;
  // Packed per-item operand images written by the pack kernel, each an SW128
  // K-major [BM x D] image: P_u | P_v | H = A_o^T G' | G' | T.
  static constexpr int PK_H = 2, PK_G = 3, PK_T = 4;
  static constexpr int ITEM_BYTES = 5 * P_BYTES;
  // Shared-memory plans (bytes).  Common: P_u at 0, P_v at P, X1 at 2P.
  static constexpr int OFF_PU = 0, OFF_PV = P_BYTES, OFF_X1 = 2 * P_BYTES;
  // DGRAD: two dU/dV buffers (SC = 64: one atom each; SC = 32: the two column
  // halves of one atom), reused for the T image in the epilogue; three
  // weight stages.
  static constexpr int D_S = 3 * P_BYTES;
  static constexpr int DS_BYTES = 4 * BM * SC * 2 > P_BYTES ? 4 * BM * SC * 2 : P_BYTES;
  static constexpr int D_NST = 3;
  // At d = 64 a channel group's weights (48 KB per role) stay resident in
  // shared memory, one slot per sub-chunk, and are loaded again only when a
  // CTA moves to another channel group; DGRAD then also has a T region of its
  // own so that T is loaded ahead of the epilogue.
  static constexpr bool RES = D == 64;
  static constexpr int D_W = D_S + DS_BYTES;
  static constexpr int D_T = D_W + (RES ? NSUB : D_NST) * A_BYTES;
  static constexpr int D_T_END = D_T + (RES ? P_BYTES : 0);
  // DGRAD epilogue: per compute warp an f32 staging tile of 8 rows x 64
  // channels (row stride 72) for the dX stores.
  static constexpr int D_ST_LD = 72;
  static constexpr int D_STG_WARP = 8 * D_ST_LD * 4;
  static constexpr int D_STG = D_T_END;
  static constexpr int D_END = D_STG + 8 * D_STG_WARP;
  static constexpr int D_TT = RES ? D_T : D_S;              // where the epilogue reads T
  // UV: item buffers (two at d = 64), dU_h | dV_h for 128 features, two stages.
  static constexpr int U_NB = D == 64 ? 2 : 1;
  static constexpr int U_S = U_NB * 3 * P_BYTES;
  static constexpr int U_W = U_S + 4 * Z_BYTES;
  static constexpr int U_END = U_W + 2 * A_BYTES;
  // O: P_u | P_v | H | G', the Z of one 128-feature pair (M_o reads it
  // directly; Y staging in the epilogue), two [B_u | B_v] stages, two B_o stages.
  static constexpr int O_G = 3 * P_BYTES;                    // G' (H sits at OFF_X1)
  static constexpr int O_ZP = 4 * P_BYTES;                   // Z of one 128-feature pair
  static constexpr int O_W1 = O_ZP + 2 * Z_BYTES;
  static constexpr int O_BO = O_W1 + 4 * SUB_BYTES;
  static constexpr int O_END = O_BO + 2 * BO_BYTES;
  static constexpr int MAX_END = D_END > U_END ? (D_END > O_END ? D_END : O_END) : (U_END > O_END ? U_END : O_END);
  static constexpr int OFF_META = MAX_END;                   // row[BM], ch[D], cont
  static constexpr int META_BYTES = (BM + D + 4) * 4;
  static constexpr int OFF_BAR = OFF_META + META_BYTES;
  static constexpr int NBARS = 28;
  static constexpr int BAR_BYTES = NBARS * 8 + 16;
  static constexpr int SMEM = OFF_BAR + BAR_BYTES + 1024;
  static_assert(SMEM <= 232448, "shared memory budget");
  static_assert(STG_BYTES <= 2 * Z_BYTES, "Y staging fits the (A_o Z) buffer");
  static_assert(!RES || (NSUB <= 2 && NSUB_UV <= 2 && RD / 64 <= 2), "resident weights fit the slots");
  // TMEM columns.  DGRAD / UV: U/V/dZ buffer b at b * 3SC; O: U/V buffer b at
  // b * 2SC, Y at 4SC.
  static constexpr int T_BUF3 = 3 * SC, T_BUF2 = 2 * SC;
  static constexpr int T_DPU = TMEM_COLS - 2 * D, T_DPV = TMEM_COLS - D;    // DGRAD
  static constexpr int T_ACCU = TMEM_COLS - 2 * D, T_ACCV = TMEM_COLS - D;  // UV
  static constexpr int T_Y = 4 * SC, T_ACCO = TMEM_COLS - NH * D;           // O
  static_assert(2 * T_BUF3 <= T_DPU, "TMEM budget (DGRAD / UV)");
  static_assert(T_Y + D <= T_ACCO, "TMEM budget (O)");
};

// Grid plan and workspace layout (bytes).
template <int D>
struct BPlan {
  int nD, nUVq, nOq, nH, grid;
  size_t img, amat, gg, nw, contig, pdA, pdAo, puv, po, mo, dxn, packed, total;
  BPlan(const Prob& p, bool block, int sms) {
    using C = BCfg<D>;
    nH = C::NH;
    // Split one wave of CTAs across the roles so that the slowest role
    // finishes first: each role's time is its items per CTA times its
    // steady-state time per item (us per item; UV per 128-feature half),
    // measured on B200 from per-CTA start / end timestamps of the role kernel
    // at B = 128: DGRAD 4.9, UV 2.97, O 3.5 at d = 64; 17.8, 7.75, 14.5 at
    // d = 128.  DGRAD's dX stores of channel groups with stride > 1 (radix
    // levels 1, 2) take about 11% longer.  The split is a pure function of the
    // shape and the SM count, so the weight-gradient partials (one per CTA,
    // summed in a fixed order) and hence the results are the same on every
    // run.  Every split of one wave is tried.
    const double tD = (D == 64 ? 4.9 : 17.8) * (p.chs > 1 ? 1.11 : 1.0);
    const double tU = D == 64 ? 2.97 : 7.75, tO = D == 64 ? 3.5 : 14.5;
    const int64_t nMB = (p.BQ() + 7) / 8;
    // The search is a few thousand steps; its result is kept per shape.
    static std::mutex mu;
    static std::map<std::array<int64_t, 5>, std::pair<int, int>> memo;
    const std::array<int64_t, 5> key{nMB, p.Qc, nH, sms, p.chs > 1 ? 1 : 0};
    {
      std::lock_guard<std::mutex> lk(mu);
      auto f = memo.find(key);
      if (f != memo.end()) {
        nUVq = f->second.first;
        nOq = f->second.second;
      } else {
        double best = -1.0;
        nUVq = nOq = 1;
        for (int u = 1; u <= nMB && nH * p.Qc * u + p.Qc + 1 <= sms; ++u)
          for (int o = 1; o <= nMB && nH * p.Qc * u + p.Qc * o + 1 <= sms; ++o) {
            const int64_t d = std::min<int64_t>(sms - nH * p.Qc * u - p.Qc * o, nMB * p.Qc);
            const double t = std::max({tD * (double)((nMB * p.Qc + d - 1) / d),
                                       tU * (double)((nMB + u - 1) / u), tO * (double)((nMB + o - 1) / o)});
            if (best < 0.0 || t < best) {
              best = t;
              nUVq = u;
              nOq = o;
            }
          }
        memo.emplace(key, std::make_pair(nUVq, nOq));
      }
    }
    nD = std::max(1, sms - nH * p.Qc * nUVq - p.Qc * nOq);
    nD = (int)std::min<int64_t>(nD, nMB * p.Qc);
    grid = nD + nH * p.Qc * nUVq + p.Qc * nOq;
    size_t o = 0;
    auto take = [&](size_t n) { size_t r = o; o = (o + n + 255) / 256 * 256; return r; };
    img = take((size_t)p.Qc * C::QC_IMG);
    amat = take(3 * 256 * 2);
    gg = take((size_t)p.Qc * D * 4);
    nw = take((size_t)p.C * 4);
    contig = take((size_t)p.Qc * 4);
    pdA = take((size_t)nD * NCOMP_WARPS * 2 * 256 * 4);
    pdAo = take((size_t)p.Qc * nOq * NCOMP_WARPS * 256 * 4);
    puv = take((size_t)nH * p.Qc * nUVq * 2 * 128 * D * 4);
    po = take((size_t)p.Qc * nOq * C::RD * D * 4);
    mo = take((size_t)p.Qc * C::RD * D * 4);
    dxn = block ? take((size_t)p.B * p.N * p.C * 2) : 0;  // 16-bit compute type
    packed = take((size_t)p.Qc * nMB * C::ITEM_BYTES);
    total = o;
  }
};

// ---------------------------------------------------------------------------
// Weight preparation (same conventions as the forward's prep kernel).
// ---------------------------------------------------------------------------
template <int D, typename TW, bool BF16>
__global__ void tc_bwd_prep_kernel(Prob p, const TW* __restrict__ au, const TW* __restrict__ av,
                                   const TW* __restrict__ ao, const TW* __restrict__ bu,
                                   const TW* __restrict__ bv, const TW* __restrict__ bo,
                                   const TW* __restrict__ gamma, const TW* __restrict__ nw_in,
                                   unsigned char* __restrict__ img, uint16_t* __restrict__ amat,
                                   float* __restrict__ gg, float* __restrict__ nw, int* __restrict__ contig) {
  using C = BCfg<D>;
  using T16 = std::conditional_t<BF16, __nv_bfloat16, __half>;
  // 32-bit indices: the divisors are compile-time constants (multiply-shift).
  constexpr int per_a = 3 * C::SC * D;  // one sub-chunk stage
  constexpr int per_qc = C::NSUB * per_a + C::RD * D;
  const int n_img = p.Qc * per_qc;
  const int stride = gridDim.x * blockDim.x;
  const int tid = blockIdx.x * blockDim.x + threadIdx.x;
  for (int i = tid; i < n_img; i += stride) {
    const int qc = i / per_qc;
    const int e = i - qc * per_qc;
    unsigned char* base = img + (int64_t)qc * C::QC_IMG;
    float v;
    uint32_t off;
    if (e < C::NSUB * per_a) {  // stage s: [B_u | B_v | B_o^T], rows = SC features n, K = D channels k
      const int s = (int)(e / per_a);
      const int r = (int)(e - s * per_a);
      const int sub = r / (C::SC * D), rr = r - sub * (C::SC * D);
      const int n = rr / D, k = rr - n * D;
      const int f = s * C::SC + n;
      if (sub == 0) v = load_as<float>(bu, ((int64_t)qc * D + k) * C::RD + f);
      else if (sub == 1) v = load_as<float>(bv, ((int64_t)qc * D + k) * C::RD + f);
      else {  // B_o^T scaled by the group's LayerScale gamma
        const int ch = p.ch[qc * D + k];
        v = ch < p.C ? load_as<float>(bo, ((int64_t)qc * C::RD + f) * D + k) * load_as<float>(gamma, ch) : 0.f;
      }
      off = (uint32_t)(s * C::A_BYTES + sub * C::SUB_BYTES) + sw128_off(n, k, C::SC);
    } else {  // chunk k: B_o rows = D channels c, K = 64 features of the chunk
      const int r = e - C::NSUB * per_a;
      const int kc = r / (64 * D), rr = r - kc * 64 * D;
      const int c = rr / 64, kf = rr - c * 64;
      v = load_as<float>(bo, ((int64_t)qc * C::RD + kc * 64 + kf) * D + c);
      off = (uint32_t)(C::NSUB * C::A_BYTES + kc * C::BO_BYTES) + sw128_off(c, kf, D);
    }
    *reinterpret_cast<T16*>(base + off) = Elem<T16>::from(v);
  }
  for (int i = tid; i < 3 * 256; i += stride) {
    const TW* src = i < 256 ? au : (i < 512 ? av : ao);
    T16 h = Elem<T16>::from(load_as<float>(src, i & 255));
    amat[i] = *reinterpret_cast<uint16_t*>(&h);
  }
  for (int i = tid; i < p.Qc * D; i += stride) {
    const int c = p.ch[i];
    gg[i] = c < p.C ? load_as<float>(gamma, c) : 0.f;
  }
  if (nw_in)
    for (int i = tid; i < p.C; i += stride) nw[i] = load_as<float>(nw_in, i);
  contig_flags<D>(p, contig);
}

__device__ __forceinline__ void comp_sync() { asm volatile("bar.sync 1, %0;" ::"n"(NCOMP) : "memory"); }

// Instruction descriptor with both operands MN-major (weight-gradient products).
__host__ __device__ constexpr uint32_t idesc_f16_mn(int M, int N, bool bf16) {
  return idesc_f16(M, N, bf16) | (1u << 15) | (1u << 16);
}

// Descriptor of an SW128 tile read MN-major: 64-element MN atoms ``lbo`` bytes
// apart, 8-row K groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sdesc_sw128_mn(uint32_t addr, uint32_t lbo) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

template <typename T>
__device__ __forceinline__ void load8v(const T* __restrict__ src, float (&v)[8]) {
  if constexpr (sizeof(T) == 2) {
    uint4 u = __ldg(reinterpret_cast<const uint4*>(src));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = unpack2<std::is_same_v<T, __nv_bfloat16>>(w[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  } else {
    float4 a = __ldg(reinterpret_cast<const float4*>(src));
    float4 b = __ldg(reinterpret_cast<const float4*>(src) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
}

struct GatherCtx {
  const int* row;   // [BM] b * N + token, or -1 for a pad row
  const int* ch;    // [D] channel indices
  int N, C;
  bool cont;        // one aligned run of channels
  int stride, c0;   // stride > 1: channels c0 + stride * k (layout_stride), else 0
};

// Gather one 64-channel half of the M-block (128 rows) into 16-bit storage.
// src element (row, ch) times (rstd[row] * nw[ch]) in x mode, times
// scale[b] * (gg[k] if given) in gradient mode.  ``sw`` selects the SW128
// K-major layout (rows BM) instead of the padded row-major staging layout.
template <typename TS, bool BF16>
__device__ __forceinline__ void gather_half(const GatherCtx& gc, const TS* __restrict__ src, int hf,
                                            const float* __restrict__ rstd, const float* __restrict__ nw,
                                            int x_dt, const float* __restrict__ scale,
                                            const float* __restrict__ ggq, unsigned char* dst, bool sw, int tid) {
  auto offs = [&](int r, int k) -> uint32_t {
    return sw ? sw128_off(r, k, BM) : (uint32_t)((r * STG_LD + (k & 63)) * 2);
  };
  if (gc.cont) {
    const int ch0 = gc.ch[0];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int unit = tid + u * NCOMP;
      const int r = unit >> 3, cj = unit & 7;
      const int k = hf * 64 + cj * 8;
      float v[8];
      const int rw = gc.row[r];
      if (rw >= 0) {
        const int64_t row = rw;
        const int ch = ch0 + k;
        load8v<TS>(src + row * gc.C + ch, v);
        if (rstd) {
          const float rs = rstd[row];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            float t = round_through(v[e] * rs, x_dt);
            v[e] = round_through(t * nw[ch + e], x_dt);
          }
        }
        const float s = scale ? scale[rw / gc.N] : 1.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] *= s * (ggq ? ggq[k + e] : 1.f);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = 0.f;
      }
      uint4 w;
      w.x = pack2<BF16>(v[0], v[1]);
      w.y = pack2<BF16>(v[2], v[3]);
      w.z = pack2<BF16>(v[4], v[5]);
      w.w = pack2<BF16>(v[6], v[7]);
      *reinterpret_cast<uint4*>(dst + offs(r, k)) = w;
    }
  } else {
    for (int e = tid; e < BM * 64; e += NCOMP) {
      const int r = e >> 6, k = hf * 64 + (e & 63);
      const int rw = gc.row[r], ch = gc.ch[k];
      float v = 0.f;
      if (rw >= 0 && ch < gc.C) {
        const int64_t row = rw;
        v = load_as<float>(src, row * gc.C + ch);
        if (rstd) {
          v = round_through(v * rstd[row], x_dt);
          v = round_through(v * nw[ch], x_dt);
        }
        v *= (scale ? scale[rw / gc.N] : 1.f) * (ggq ? ggq[k] : 1.f);
      }
      const uint32_t pk = pack2<BF16>(v, 0.f);
      *reinterpret_cast<uint16_t*>(dst + offs(r, k)) = (uint16_t)(pk & 0xFFFF);
    }
  }
}

// Register-staged gather of NHF 64-channel halves (contiguous channel runs):
// rows_issue() starts every load of the M-block at once; rows_store() later
// converts one half and writes it out, so one memory round trip covers the
// whole item.
template <typename TS, int NHF>
struct RowRegs {
  static constexpr int VW = sizeof(TS) == 2 ? 1 : 2;  // 16-byte vectors per 8 elements
  uint4 v[NHF][4][VW];
  float rs[4];  // per-unit row factor: rstd (x) or drop-path scale (dOut)
};

template <typename TS, int NHF>
__device__ __forceinline__ void rows_issue(RowRegs<TS, NHF>& R, const GatherCtx& gc, const TS* __restrict__ src,
                                           int hf0, const float* __restrict__ rstd, const float* __restrict__ scale,
                                           int tid) {
  const int ch0 = gc.ch[0];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int unit = tid + u * NCOMP;
    const int r = unit >> 3, cj = unit & 7;
    // Pad rows load row 0 (always valid) and are zeroed in rows_store; no
    // loaded value is used here, so the loads stay in flight.
    const int rw = gc.row[r] >= 0 ? gc.row[r] : 0;
#pragma unroll
    for (int h = 0; h < NHF; ++h) {
      const uint4* p = reinterpret_cast<const uint4*>(src + (int64_t)rw * gc.C + ch0 + (hf0 + h) * 64 + cj * 8);
#pragma unroll
      for (int vv = 0; vv < RowRegs<TS, NHF>::VW; ++vv) R.v[h][u][vv] = __ldg(p + vv);
    }
    R.rs[u] = rstd ? rstd[rw] : (scale ? scale[rw / gc.N] : 1.f);
  }
}

// x mode (nw != null or rstd given): round(round(v * rstd) * nw[ch]); gradient
// mode: v * scale * ggq[k].  ``hf`` is the absolute half (channel offset).
template <typename TS, int NHF, bool BF16>
__device__ __forceinline__ void rows_store(const RowRegs<TS, NHF>& R, int h, int hf, const GatherCtx& gc,
                                           unsigned char* dst, bool sw, bool xnorm, const float* __restrict__ nw,
                                           const float* __restrict__ ggq, int x_dt, int tid) {
  const int ch0 = gc.ch[0];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int unit = tid + u * NCOMP;
    const int r = unit >> 3, cj = unit & 7;
    const int k = hf * 64 + cj * 8;
    float v[8];
    if constexpr (sizeof(TS) == 2) {
      const uint32_t w[4] = {R.v[h][u][0].x, R.v[h][u][0].y, R.v[h][u][0].z, R.v[h][u][0].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float2 f = unpack2<std::is_same_v<TS, __nv_bfloat16>>(w[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
      }
    } else {
#pragma unroll
      for (int vv = 0; vv < 2; ++vv) {
        v[4 * vv + 0] = __uint_as_float(R.v[h][u][vv].x);
        v[4 * vv + 1] = __uint_as_float(R.v[h][u][vv].y);
        v[4 * vv + 2] = __uint_as_float(R.v[h][u][vv].z);
        v[4 * vv + 3] = __uint_as_float(R.v[h][u][vv].w);
      }
    }
    if (xnorm) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float t = round_through(v[e] * R.rs[u], x_dt);
        v[e] = round_through(t * nw[ch0 + k + e], x_dt);
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] *= R.rs[u] * (ggq ? ggq[k + e] : 1.f);
    }
    if (gc.row[r] < 0) {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = 0.f;
    }
    uint4 w;
    w.x = pack2<BF16>(v[0], v[1]);
    w.y = pack2<BF16>(v[2], v[3]);
    w.z = pack2<BF16>(v[4], v[5]);
    w.w = pack2<BF16>(v[6], v[7]);
    const uint32_t off = sw ? sw128_off(r, k, BM) : (uint32_t)((r * STG_LD + cj * 8) * 2);
    *reinterpret_cast<uint4*>(dst + off) = w;
  }
}

// Gather of one 64-channel half of a strided group (channels c0 + S k,
// S = gc.stride in {2, 4, 8}, c0 < S) into the row-major staging layout.
// The half's channels lie in the aligned span [64 S hf, 64 S (hf + 1)) of the
// row: consecutive threads read consecutive 16-byte vectors of it (the
// sibling groups of the same rows read the rest, so the extra bytes come from
// L2), and each vector contributes its 8 / S elements of this group.  Same
// arithmetic as rows_store: x mode round(round(v * rstd) * nw[c]), gradient
// mode v * scale[b]; pad rows are zero.
template <typename TS, bool BF16, int S, int UPP>
__device__ __forceinline__ void gather_half_strided_t(const GatherCtx& gc, const TS* __restrict__ src, int hf,
                                                      bool xnorm, const float* __restrict__ rstd,
                                                      const float* __restrict__ nw, int x_dt,
                                                      const float* __restrict__ scale, unsigned char* stg,
                                                      int tid) {
  constexpr int VW = sizeof(TS) == 2 ? 1 : 2;  // 16-byte vectors per 8 elements
  constexpr int VPR = 8 * S;                   // vectors of 8 elements per row span
  constexpr int UNITS = BM * VPR;              // 4 S units per thread
  const int c0 = gc.c0;
  const int64_t span0 = (int64_t)S * hf * 64;
#pragma unroll 1
  for (int u0 = 0; u0 < UNITS; u0 += UPP * NCOMP) {
    uint4 v[UPP][VW];
    float rs[UPP];
#pragma unroll
    for (int j = 0; j < UPP; ++j) {
      const int unit = u0 + j * NCOMP + tid;
      const int r = unit / VPR, vi = unit % VPR;
      // Pad rows load row 0 (always valid) and are zeroed below.
      const int rw = gc.row[r] >= 0 ? gc.row[r] : 0;
      const uint4* p = reinterpret_cast<const uint4*>(src + (int64_t)rw * gc.C + span0 + vi * 8);
#pragma unroll
      for (int w = 0; w < VW; ++w) v[j][w] = __ldg(p + w);
      rs[j] = xnorm ? rstd[rw] : (scale ? scale[rw / gc.N] : 1.f);
    }
#pragma unroll
    for (int j = 0; j < UPP; ++j) {
      const int unit = u0 + j * NCOMP + tid;
      const int r = unit / VPR, vi = unit % VPR;
      const bool pad = gc.row[r] < 0;
      constexpr int NT = 8 / S;  // this group's elements in the vector
      float fv[NT];
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const int i = c0 + S * t;
        const uint32_t w32 = (i >> 1) == 0 ? v[j][0].x : (i >> 1) == 1 ? v[j][0].y : (i >> 1) == 2 ? v[j][0].z : v[j][0].w;
        float f;
        if constexpr (sizeof(TS) == 2) {
          const float2 t2 = unpack2<std::is_same_v<TS, __nv_bfloat16>>(w32);
          f = (i & 1) ? t2.y : t2.x;
        } else {
          const uint4 q = i < 4 ? v[j][0] : v[j][VW - 1];  // selects, no dynamic register indexing
          const int e = i & 3;
          f = __uint_as_float(e == 0 ? q.x : e == 1 ? q.y : e == 2 ? q.z : q.w);
        }
        if (xnorm) {
          f = round_through(f * rs[j], x_dt);
          f = round_through(f * nw[span0 + vi * 8 + i], x_dt);
        } else {
          f *= rs[j];
        }
        fv[t] = pad ? 0.f : f;
      }
      // The NT consecutive k of this vector in one store (8, 4 or 2 bytes).
      unsigned char* dst = stg + (r * STG_LD + vi * NT) * 2;
      if constexpr (NT == 4) {
        *reinterpret_cast<uint2*>(dst) = make_uint2(pack2<BF16>(fv[0], fv[1]), pack2<BF16>(fv[2], fv[3]));
      } else if constexpr (NT == 2) {
        *reinterpret_cast<uint32_t*>(dst) = pack2<BF16>(fv[0], fv[1]);
      } else {
        *reinterpret_cast<uint16_t*>(dst) = (uint16_t)(pack2<BF16>(fv[0], 0.f) & 0xFFFF);
      }
    }
  }
}

// Units per thread whose 16-byte loads are in flight together: eight for a
// 16-bit source, except in the forward pre-pass at stride 2, whose smaller
// CTAs run more per SM (measured faster with four); f32 sources four
// (register budget).
template <typename TS, bool BF16, bool FWD>
__device__ __forceinline__ void gather_half_strided(const GatherCtx& gc, const TS* __restrict__ src, int hf,
                                                    bool xnorm, const float* __restrict__ rstd,
                                                    const float* __restrict__ nw, int x_dt,
                                                    const float* __restrict__ scale, unsigned char* stg, int tid) {
  switch (gc.stride) {
    case 2: gather_half_strided_t<TS, BF16, 2, (sizeof(TS) == 2 && !FWD) ? 8 : 4>(gc, src, hf, xnorm, rstd, nw, x_dt, scale, stg, tid); break;
    case 4: gather_half_strided_t<TS, BF16, 4, sizeof(TS) == 2 ? 8 : 4>(gc, src, hf, xnorm, rstd, nw, x_dt, scale, stg, tid); break;
    default: gather_half_strided_t<TS, BF16, 8, sizeof(TS) == 2 ? 8 : 4>(gc, src, hf, xnorm, rstd, nw, x_dt, scale, stg, tid); break;
  }
}

// Token mix of one 64-channel half: dst[rows of tile ``warp``] = A * staging,
// written in SW128 K-major layout at channel offset hf*64.
template <bool BF16>
__device__ __forceinline__ void mix_half(uint32_t aStg, const uint32_t (&fa)[4], unsigned char* dst, int hf,
                                         int warp, int lane, const float* colscale = nullptr) {
  const int g = lane >> 2, t4 = lane & 3;
#pragma unroll
  for (int np = 0; np < 4; ++np) {
    uint32_t b0, b1, b2, b3;
    ldsm_x4_trans(aStg + ((warp * 16 + (lane & 15)) * STG_LD + np * 16 + (lane >> 4) * 8) * 2, b0, b1, b2, b3);
    float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
    mma16816<BF16>(c0, fa, b0, b1);
    mma16816<BF16>(c1, fa, b2, b3);
    const int r0 = warp * 16 + g, k0 = hf * 64 + np * 16 + 2 * t4;
    if (colscale) {
      const float s0 = colscale[k0], s1 = colscale[k0 + 1], s2 = colscale[k0 + 8], s3 = colscale[k0 + 9];
      c0[0] *= s0; c0[1] *= s1; c0[2] *= s0; c0[3] *= s1;
      c1[0] *= s2; c1[1] *= s3; c1[2] *= s2; c1[3] *= s3;
    }
    *reinterpret_cast<uint32_t*>(dst + sw128_off(r0, k0, BM)) = pack2<BF16>(c0[0], c0[1]);
    *reinterpret_cast<uint32_t*>(dst + sw128_off(r0 + 8, k0, BM)) = pack2<BF16>(c0[2], c0[3]);
    *reinterpret_cast<uint32_t*>(dst + sw128_off(r0, k0 + 8, BM)) = pack2<BF16>(c1[0], c1[1]);
    *reinterpret_cast<uint32_t*>(dst + sw128_off(r0 + 8, k0 + 8, BM)) = pack2<BF16>(c1[2], c1[3]);
  }
}

// acc[nb] (16x8 blocks nb = 0,1 of a 16x16 result) += L[16 x 64] * R[16 x 64]^T
// for the tile of ``warp``.  L rows come from ``lrow(row, col)`` addresses,
// R rows from ``rrow(row, col)`` (both 16-bit, 16-byte chunks contiguous).
template <bool BF16, typename LA, typename RA>
__device__ __forceinline__ void gram16(float (&acc)[2][4], LA lrow, RA rrow, int lane) {
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    const int k0 = ks * 16;
    uint32_t a[4], b[4];
    ldsm_x4(lrow((lane & 7) + ((lane >> 3) & 1) * 8, k0 + (lane >> 4) * 8), a[0], a[1], a[2], a[3]);
    ldsm_x4(rrow((lane & 7) + (lane >> 4) * 8, k0 + ((lane >> 3) & 1) * 8), b[0], b[1], b[2], b[3]);
    mma16816<BF16>(acc[0], a, b[0], b[1]);
    mma16816<BF16>(acc[1], a, b[2], b[3]);
  }
}

struct BwdArgs {
  Prob p;
  const void* x;
  const void* dout;
  const float* rstd;
  const float* scale;
  int x_dt;
  const unsigned char* img;
  const uint16_t* amat;
  const float* gg;
  const float* nw;
  const int* contig;
  int vec_ok;
  unsigned char* packed;  // [items][5][BM x D] SW128 operand images
  void* dx;       // operator mode: x dtype
  void* dxn;      // block mode: gradient w.r.t. the normalised input, 16-bit compute type
  float* pdA;     // [nD][8][2][256]
  float* pdAo;    // [Qc*nOq][8][256]
  float* puv;     // [nH*Qc*nUVq][2][128][D]
  float* po;      // [Qc*nOq][RD][D]
  int nD, nUVq, nOq, nH;
  int* fault;         // device fault word (bounded waits that gave up)
  uint32_t probe_ns;  // wait-timeout self-check (0: off)
};

// ---------------------------------------------------------------------------
// Pack kernel: gathers one M-block (128 token rows) of x (RMS-normalised in
// block mode) and of dOut through the route tables and writes the operand
// images the backward roles consume, once per item:
//   P_u = A_u T, P_v = A_v T, H = A_o^T G', G', T
// (G' = mask * drop-path scale * dOut).  Many small CTAs per SM hide the
// gather latency that a single persistent CTA could not.  Each 64-channel
// half of an image is one 16 KB SW128 atom; it is built in shared memory and
// written with one bulk copy, so the global writes are full lines.
// ---------------------------------------------------------------------------
// FWD: the forward's pre-pass; writes only [P_u | P_v] per item (2 images).
template <int D, bool BF16, typename TX, typename TO, bool FWD = false>
__global__ void __launch_bounds__(NCOMP) tc_pack_kernel(BwdArgs a) {
  using C = BCfg<D>;
  constexpr int ATOM = BM * 128;  // one 64-channel half of an operand image
  const Prob& p = a.p;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>(((uintptr_t)smem_raw + 127) & ~(uintptr_t)127);
  // The forward mode needs no third atom: a smaller footprint lets more
  // CTAs share an SM.
  constexpr int NATOM = FWD ? 2 : 3;
  unsigned char* atom1 = sm;             // P_u, then H
  unsigned char* atom2 = sm + ATOM;      // P_v
  unsigned char* atom0 = sm + 2 * ATOM;  // T, then G' (not in the forward mode)
  unsigned char* stg = sm + NATOM * ATOM;  // gathered half, row-major
  int* sRow = reinterpret_cast<int*>(stg + STG_BYTES);
  int* sCh = sRow + BM;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int64_t BQ = (int64_t)p.B * p.Qs;
  const int nMB = (int)((BQ + 7) / 8);
  // CTAs run M-block-major (all channel groups of one M-block in a row), so
  // the groups of a token row are gathered close together in time and share
  // DRAM pages; the images stay in channel-group-major item order.
  const int mb = (int)(blockIdx.x / p.Qc), qc = (int)(blockIdx.x - (int64_t)mb * p.Qc);
  const int64_t item = (int64_t)qc * nMB + mb;
  for (int r = tid; r < BM; r += NCOMP) {
    const int64_t t = (int64_t)mb * 8 + (r >> 4);
    int rw = -1;
    if (t < BQ) {
      const int b = (int)(t / p.Qs);
      const int tok = p.tok[(t - (int64_t)b * p.Qs) * 16 + (r & 15)];
      rw = tok < p.N ? b * p.N + tok : -1;
    }
    sRow[r] = rw;
  }
  for (int k = tid; k < D; k += NCOMP) sCh[k] = p.ch[qc * D + k];
  __syncthreads();
  const int lay = a.contig[qc];
  const int lst = a.vec_ok ? layout_stride(lay) : 0;
  GatherCtx gc{sRow, sCh, p.N, p.C, lst == 1, lst > 1 ? lst : 0, layout_c0(lay)};
  // FWD item: [P_u | P_v | output row of each of the BM token rows (int32, -1: none)].
  unsigned char* out = a.packed + item * (FWD ? 2 * C::P_BYTES + BM * 4 : C::ITEM_BYTES);
  const uint32_t aStg = smem_u32(stg);
  const TX* x = (const TX*)a.x;
  const TO* dout = (const TO*)a.dout;
  // staging (row-major) -> SW128 atom in shared memory
  auto to_atom = [&](unsigned char* atom) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int unit = tid + u * NCOMP;
      const int r = unit >> 3, cj = unit & 7;
      const uint4 v = *reinterpret_cast<const uint4*>(stg + (r * STG_LD + cj * 8) * 2);
      *reinterpret_cast<uint4*>(atom + sw128_off(r, cj * 8, BM)) = v;
    }
  };
  // Atoms are byte-identical to the global image halves: one bulk store each.
  auto atoms_ready = [&]() {
    fence_proxy_async_smem();
    __syncthreads();
  };
  auto atoms_free = [&]() {
    if (tid == 0) bulk_wait_read();
    __syncthreads();
  };
  for (int hf = 0; hf < D / 64; ++hf) {
    RowRegs<TO, 1> rg;
    if (gc.cont) {
      RowRegs<TX, 1> rx;
      rows_issue<TX, 1>(rx, gc, x, hf, a.rstd, nullptr, tid);
      if (!FWD) rows_issue<TO, 1>(rg, gc, dout, hf, nullptr, a.scale, tid);
      rows_store<TX, 1, BF16>(rx, 0, hf, gc, stg, false, a.rstd != nullptr, a.nw, nullptr, a.x_dt, tid);
    } else if (gc.stride) {
      gather_half_strided<TX, BF16, FWD>(gc, x, hf, a.rstd != nullptr, a.rstd, a.nw, a.x_dt, nullptr, stg, tid);
    } else {
      gather_half<TX, BF16>(gc, x, hf, a.rstd, a.nw, a.x_dt, nullptr, nullptr, stg, false, tid);
    }
    atoms_free();  // also publishes stg
    if (!FWD) to_atom(atom0);
    {
      uint32_t f[4];
      load_afrag(a.amat, false, g, t4, f);
      mix_half<BF16>(aStg, f, atom1, 0, warp, lane);
      load_afrag(a.amat + 256, false, g, t4, f);
      mix_half<BF16>(aStg, f, atom2, 0, warp, lane);
    }
    atoms_ready();
    if (tid == 0) {
      if (!FWD) bulk_s2g(out + C::PK_T * C::P_BYTES + hf * ATOM, atom0, ATOM);
      if (FWD && hf == 0) bulk_s2g(out + 2 * C::P_BYTES, sRow, BM * 4);
      bulk_s2g(out + hf * ATOM, atom1, ATOM);
      bulk_s2g(out + C::P_BYTES + hf * ATOM, atom2, ATOM);
      bulk_commit();
    }
    if (FWD) continue;
    if (gc.cont) rows_store<TO, 1, BF16>(rg, 0, hf, gc, stg, false, false, nullptr, nullptr, 0, tid);
    else if (gc.stride) gather_half_strided<TO, BF16, FWD>(gc, dout, hf, false, nullptr, nullptr, 0, a.scale, stg, tid);
    else gather_half<TO, BF16>(gc, dout, hf, nullptr, nullptr, 0, a.scale, nullptr, stg, false, tid);
    atoms_free();
    to_atom(atom0);
    {
      uint32_t f[4];
      load_afrag(a.amat + 512, true, g, t4, f);
      mix_half<BF16>(aStg, f, atom1, 0, warp, lane);  // H = A_o^T G'
    }
    atoms_ready();
    if (tid == 0) {
      bulk_s2g(out + C::PK_G * C::P_BYTES + hf * ATOM, atom0, ATOM);
      bulk_s2g(out + C::PK_H * C::P_BYTES + hf * ATOM, atom1, ATOM);
      bulk_commit();
    }
  }
  if (tid == 0) bulk_wait_all();
}

// ---------------------------------------------------------------------------
// Role kernel (see the file header).  The feature dimension is walked in
// sub-chunks of SC features.  The tensor pipe fills one TMEM buffer with the
// next sub-chunk's U/V(/dZ) while the compute warps turn the other buffer
// into elementwise outputs; item operands and weight stages arrive by bulk
// copies issued ahead of use by the producer warp.
// ---------------------------------------------------------------------------
template <int D, bool BF16, typename TX, typename TO>
__global__ void __launch_bounds__(TC_THREADS, 1) tc_bwd_kernel(BwdArgs a) {
  using C = BCfg<D>;
  using T16 = std::conditional_t<BF16, __nv_bfloat16, __half>;
  constexpr int SC = C::SC;
  constexpr int HC = SC / 2;            // columns of a sub-chunk per compute thread
  constexpr bool HALVES = SC == 32;     // two buffers share one 64-column atom
  constexpr int NB_UV = C::U_NB;
  const Prob& p = a.p;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  int* sRow = reinterpret_cast<int*>(sm + C::OFF_META);
  int* sCh = sRow + BM;
  volatile int* sCont = sCh + D;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + C::OFF_BAR);
  uint64_t* bar_p = bars + 0;     // [2] item operands of item buffer i loaded (tx)
  uint64_t* bar_a = bars + 2;     // [2] U/V(/dZ) of TMEM buffer b computed (commit)
  uint64_t* bar_du = bars + 4;    // [2] compute done with TMEM buffer b, its outputs in smem
  uint64_t* bar_b = bars + 6;     // [2] DGRAD: dP read dU/dV buffer b; O: Y read Z buffer b (commit)
  uint64_t* bar_wf = bars + 8;    // [3] weight stage loaded (tx)
  uint64_t* bar_we = bars + 11;   // [3] DGRAD: weight stage no longer read (commit)
  uint64_t* bar_bo = bars + 14;   // [2] O: B_o stage loaded (tx)
  uint64_t* bar_boe = bars + 16;  // [2] O: B_o stage no longer read (commit)
  uint64_t* bar_pf = bars + 18;   // DGRAD, O: item operands no longer read (commit)
  uint64_t* bar_tf = bars + 19;   // DGRAD: last dP of the item done (commit)
  uint64_t* bar_t = bars + 20;    // DGRAD: T image loaded (tx)
  uint64_t* bar_w = bars + 21;    // UV: products of an item done; O: M_o of a pair done (commit)
  uint64_t* bar_yd = bars + 23;   // O: Y of the item complete (commit)
  uint64_t* bar_epd = bars + 24;  // epilogue done (DGRAD: T; O: H, G' and the staging buffer)
  uint64_t* bar_gl = bars + 25;   // O: H and G' loaded (tx)
  uint64_t* bar_probe = bars + 26;  // wait-timeout self-check: nothing arrives on it
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(bars + C::NBARS);
  volatile int* sAbort = reinterpret_cast<volatile int*>(sTmem + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t BQ = (int64_t)p.B * p.Qs;
  const int nMB = (int)((BQ + 7) / 8);

  // ---- role of this CTA and its item range
  int role, h = 0, wslot = 0;
  int64_t it0 = 0, it_step = 1, n_items = 0;
  {
    const int b = blockIdx.x;
    const int nUV = a.nH * p.Qc * a.nUVq;
    if (b < a.nD) {
      role = R_DGRAD;
      it0 = b;
      it_step = a.nD;
      const int64_t items = (int64_t)p.Qc * nMB;
      n_items = items > b ? (items - 1 - b) / a.nD + 1 : 0;
    } else {
      int local, nq;
      if (b < a.nD + nUV) {
        role = R_UV;
        local = b - a.nD;
        h = local / (p.Qc * a.nUVq);
        local -= h * p.Qc * a.nUVq;
        nq = a.nUVq;
        wslot = (h * p.Qc + local / nq) * nq + local % nq;
      } else {
        role = R_O;
        local = b - a.nD - nUV;
        nq = a.nOq;
        wslot = local;
      }
      const int qc_fix = local / nq;
      const int j = local % nq;
      const int64_t m0 = (int64_t)nMB * j / nq, m1 = (int64_t)nMB * (j + 1) / nq;
      it0 = (int64_t)qc_fix * nMB + m0;
      it_step = 1;
      n_items = m1 - m0;
    }
  }
  const int nsub = role == R_UV ? C::NSUB_UV : C::NSUB;
  const int q_base = role == R_UV ? h * C::NSUB_UV : 0;  // first sub-chunk of the role's features
  // Each CTA walks its sub-chunks from a different starting point so that the
  // CTAs of one role do not all fetch the same weight stage at once (the O
  // role rotates by whole 128-feature pairs).
  const int rot = role == R_O ? (int)(blockIdx.x % C::NH) * (128 / C::SC) : (int)(blockIdx.x % nsub);
  auto sub_of = [&](int j) { return (j + rot) % nsub; };
  const int nit = (int)n_items;
  const int total = nit * nsub;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar_p + i, 1);
      mbar_init(bar_a + i, 1);
      mbar_init(bar_du + i, NCOMP);
      mbar_init(bar_b + i, 1);
      mbar_init(bar_bo + i, 1);
      mbar_init(bar_boe + i, 1);
    }
    for (int i = 0; i < 3; ++i) {
      mbar_init(bar_wf + i, 1);
      mbar_init(bar_we + i, 1);
    }
    mbar_init(bar_pf, 1);
    mbar_init(bar_tf, 1);
    mbar_init(bar_t, 1);
    mbar_init(bar_w, 1);
    mbar_init(bar_yd, 1);
    mbar_init(bar_epd, NCOMP);
    mbar_init(bar_gl, 1);
    mbar_init(bar_probe, 1);
    *sAbort = 0;
    fence_mbar_init();
    wait_probe(bar_probe, sAbort, a.probe_ns);
  }
  if (warp == MMA_WARP) tmem_alloc(sTmem, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *sTmem;

  auto item_of = [&](int it) { return it0 + (int64_t)it * it_step; };
  auto item_src = [&](int it) { return a.packed + item_of(it) * C::ITEM_BYTES; };
  auto qimg = [&](int c) { return a.img + (item_of(c / nsub) / nMB) * C::QC_IMG; };
  auto stage_src = [&](int c) { return qimg(c) + (int64_t)(q_base + sub_of(c % nsub)) * C::A_BYTES; };
  auto bo_src = [&](int c) {
    return qimg(c) + (int64_t)C::NSUB * C::A_BYTES + (int64_t)(sub_of(c % nsub) / C::SPC) * C::BO_BYTES;
  };
  // Double-buffered 64-row-block operands (dU/dV for DGRAD, Z for O): byte
  // offset of buffer b's atom and its first column.
  auto buf_atom = [&](int b, int atoms_per_buf) -> uint32_t {
    return HALVES ? 0u : (uint32_t)(b * atoms_per_buf * C::Z_BYTES);
  };
  auto buf_col = [&](int b) { return HALVES ? b * 32 : 0; };

  if (*sAbort) {
    // The wait-timeout self-check ran out before any work was issued.
  } else if (warp == PROD_WARP) {
    // ------------------------------------------------ producer (bulk copies)
    if (lane == 0 && nit > 0) {
      if (role == R_DGRAD) {
        auto load_item = [&](int it) {
          mbar_arrive_expect_tx(bar_p, 3 * C::P_BYTES);
          bulk_g2s(sm, item_src(it), 3 * C::P_BYTES, bar_p);
        };
        auto load_w = [&](int c) {
          const int st = c % C::D_NST;
          mbar_arrive_expect_tx(bar_wf + st, C::A_BYTES);
          bulk_g2s(sm + C::D_W + st * C::A_BYTES, stage_src(c), C::A_BYTES, bar_wf + st);
        };
        auto load_t = [&](int it) {
          mbar_arrive_expect_tx(bar_t, C::P_BYTES);
          bulk_g2s(sm + C::D_TT, item_src(it) + C::PK_T * C::P_BYTES, C::P_BYTES, bar_t);
        };
        load_item(0);
        if constexpr (C::RES) {
          // All sub-chunk stages of the item's channel group, in one copy.
          auto load_all = [&](int it) {
            mbar_arrive_expect_tx(bar_wf, C::NSUB * C::A_BYTES);
            bulk_g2s(sm + C::D_W, qimg(it * nsub), C::NSUB * C::A_BYTES, bar_wf);
          };
          load_all(0);
          load_t(0);
          int epoch = 0;
          for (int it = 0; it + 1 < nit && !*sAbort; ++it) {
            if (mbar_wait(bar_pf, it & 1, sAbort)) {
              load_item(it + 1);
            }
            if (item_of(it + 1) / nMB != item_of(it) / nMB && mbar_wait(bar_we, epoch & 1, sAbort)) {
              ++epoch;
              load_all(it + 1);
            }
            if (mbar_wait(bar_epd, it & 1, sAbort)) {
              load_t(it + 1);
            }
          }
        } else {
          for (int c = 0; c < C::D_NST && c < total; ++c) load_w(c);
          for (int c = 0; c < total && !*sAbort; ++c) {
            const int it = c / nsub, j = c - it * nsub;
            if (j == nsub - 1 && it + 1 < nit && mbar_wait(bar_pf, it & 1, sAbort)) {
              load_item(it + 1);
            }
            if (c + C::D_NST < total && mbar_wait(bar_we + c % C::D_NST, (c / C::D_NST) & 1, sAbort))
              load_w(c + C::D_NST);
            if (j == nsub - 1 && mbar_wait(bar_tf, it & 1, sAbort)) {
              load_t(it);
            }
          }
        }
      } else if (role == R_UV) {
        auto load_item = [&](int it) {
          const int bf = it % NB_UV;
          mbar_arrive_expect_tx(bar_p + bf, 3 * C::P_BYTES);
          bulk_g2s(sm + bf * 3 * C::P_BYTES, item_src(it), 3 * C::P_BYTES, bar_p + bf);
        };
        auto load_w = [&](int c) {
          const int st = c & 1;
          mbar_arrive_expect_tx(bar_wf + st, C::A_BYTES);
          bulk_g2s(sm + C::U_W + st * C::A_BYTES, stage_src(c), C::A_BYTES, bar_wf + st);
        };
        for (int it = 0; it < NB_UV && it < nit; ++it) load_item(it);
        if constexpr (C::RES) {  // the half's stages, once (the group never changes)
          mbar_arrive_expect_tx(bar_wf, C::NSUB_UV * C::A_BYTES);
          bulk_g2s(sm + C::U_W, qimg(0) + (int64_t)q_base * C::A_BYTES, C::NSUB_UV * C::A_BYTES, bar_wf);
        } else {
          load_w(0);
          if (total > 1) load_w(1);
        }
        for (int c = 0; c < total && !*sAbort; ++c) {
          const int it = c / nsub, j = c - it * nsub;
          if (!C::RES && c + 2 < total && mbar_wait(bar_a + (c & 1), (c >> 1) & 1, sAbort)) load_w(c + 2);
          if (j == nsub - 1 && it + NB_UV < nit && mbar_wait(bar_w, it & 1, sAbort)) {
            load_item(it + NB_UV);
          }
        }
      } else {
        const int nck = total / C::SPC;
        auto load_p = [&](int it) {
          mbar_arrive_expect_tx(bar_p, 2 * C::P_BYTES);
          bulk_g2s(sm, item_src(it), 2 * C::P_BYTES, bar_p);
        };
        auto load_g = [&](int it) {  // H | G' (adjacent in the packed item)
          mbar_arrive_expect_tx(bar_gl, 2 * C::P_BYTES);
          bulk_g2s(sm + C::OFF_X1, item_src(it) + C::PK_H * C::P_BYTES, 2 * C::P_BYTES, bar_gl);
        };
        auto load_w1 = [&](int c) {
          const int st = c & 1;
          mbar_arrive_expect_tx(bar_wf + st, 2 * C::SUB_BYTES);
          bulk_g2s(sm + C::O_W1 + st * 2 * C::SUB_BYTES, stage_src(c), 2 * C::SUB_BYTES, bar_wf + st);
        };
        auto load_bo = [&](int kc) {
          const int st = kc & 1;
          mbar_arrive_expect_tx(bar_bo + st, C::BO_BYTES);
          bulk_g2s(sm + C::O_BO + st * C::BO_BYTES, bo_src(kc * C::SPC), C::BO_BYTES, bar_bo + st);
        };
        load_p(0);
        load_g(0);
        if constexpr (C::RES) {  // [B_u | B_v] of every sub-chunk and all of B_o, once
          const unsigned char* g0 = qimg(0);
          mbar_arrive_expect_tx(bar_wf, C::NSUB * 2 * C::SUB_BYTES + (C::RD / 64) * C::BO_BYTES);
          for (int sj = 0; sj < C::NSUB; ++sj)
            bulk_g2s(sm + C::O_W1 + sj * 2 * C::SUB_BYTES, g0 + (int64_t)sj * C::A_BYTES, 2 * C::SUB_BYTES, bar_wf);
          bulk_g2s(sm + C::O_BO, g0 + (int64_t)C::NSUB * C::A_BYTES, (C::RD / 64) * C::BO_BYTES, bar_wf);
        } else {
          load_w1(0);
          if (total > 1) load_w1(1);
          load_bo(0);
          if (nck > 1) load_bo(1);
        }
        for (int c = 0; c < total && !*sAbort; ++c) {
          const int it = c / nsub, j = c - it * nsub;
          if (!C::RES && c + 2 < total && mbar_wait(bar_a + (c & 1), (c >> 1) & 1, sAbort)) load_w1(c + 2);
          const bool last = j == nsub - 1 && it + 1 < nit;
          if (last && mbar_wait(bar_pf, it & 1, sAbort)) {
            load_p(it + 1);
          }
          if (!C::RES && c % C::SPC == C::SPC - 1) {
            const int kc = c / C::SPC;
            if (kc + 2 < nck && mbar_wait(bar_boe + (kc & 1), (kc >> 1) & 1, sAbort)) load_bo(kc + 2);
          }
          if (last && mbar_wait(bar_epd, it & 1, sAbort)) {
            load_g(it + 1);
          }
        }
      }
    }
  } else if (warp == MMA_WARP) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t ID_N = idesc_f16(BM, SC, BF16);
      constexpr uint32_t ID_ND = idesc_f16(BM, D, BF16);
      constexpr uint32_t ID_MN = idesc_f16_mn(BM, D, BF16);
      constexpr uint32_t ID_BMN = idesc_f16(BM, D, BF16) | (1u << 16);  // A K-major, B MN-major
      // D (+)= A * B^T over ksteps 16-element K steps, both SW128 K-major.
      auto kmma = [&](uint32_t tcol, uint32_t aA, int arows, int ka, uint32_t aB, int brows, int kb, int ksteps,
                      uint32_t id, bool acc0) {
        for (int kk = 0; kk < ksteps; ++kk)
          umma_f16(tbase + tcol, sdesc_sw128(sw128_kstep(aA, ka + kk, arows)),
                   sdesc_sw128(sw128_kstep(aB, kb + kk, brows)), id, (acc0 || kk > 0) ? 1u : 0u);
      };
      // D (+)= A^T B over the 128 tokens, A and B token-major tiles read MN-major.
      auto mnmma = [&](uint32_t tcol, uint32_t aA, uint32_t aB, bool acc0) {
        for (int kk = 0; kk < BM / 16; ++kk)
          umma_f16(tbase + tcol, sdesc_sw128_mn(aA + kk * 2048, BM * 128), sdesc_sw128_mn(aB + kk * 2048, BM * 128),
                   ID_MN, (acc0 || kk > 0) ? 1u : 0u);
      };
      const uint32_t s0 = smem_u32(sm);
      if (role == R_DGRAD) {
        const uint32_t aPu = s0 + C::OFF_PU, aPv = s0 + C::OFF_PV, aDY = s0 + C::OFF_X1;
        auto dp = [&](int x) {  // dP_u += dU_x B_u[x]^T, dP_v += dV_x B_v[x]^T
          const int bx = x & 1, jx = x % nsub;
          mbar_wait(bar_du + bx, (x >> 1) & 1, sAbort);
          tc_fence_after();
          if (!*sAbort) {
            const uint32_t aU = s0 + C::D_S + buf_atom(bx, 2), aV = aU + C::Z_BYTES;
            const uint32_t aSt = s0 + C::D_W + (C::RES ? sub_of(jx) : x % C::D_NST) * C::A_BYTES;
            const int k0 = buf_col(bx) / 16;
            for (int kk = 0; kk < SC / 16; ++kk) {
              const uint32_t acc = (jx > 0 || kk > 0) ? 1u : 0u;
              umma_f16(tbase + C::T_DPU, sdesc_sw128(sw128_kstep(aU, k0 + kk, BM)),
                       sdesc_sw128_mn(aSt + kk * 2048, SC * 128), ID_BMN, acc);
              umma_f16(tbase + C::T_DPV, sdesc_sw128(sw128_kstep(aV, k0 + kk, BM)),
                       sdesc_sw128_mn(aSt + C::SUB_BYTES + kk * 2048, SC * 128), ID_BMN, acc);
            }
          }
          umma_commit(bar_b + bx);
          if (!C::RES) umma_commit(bar_we + x % C::D_NST);
          if (jx == nsub - 1) umma_commit(bar_tf);
        };
        int c = 0, epoch = 0;
        for (int it = 0; it < nit; ++it) {
          if (c > 0) dp(c - 1);  // finish the previous item before waiting for this one's operands
          // The epilogue's warp-level MMAs share the tensor pipe: only the
          // first sub-chunk's U/V/dZ go ahead of them (the compute warps find
          // them done when the epilogue ends; the epilogue's closing barrier
          // orders the reuse of the dU/dV buffers, which hold T at d = 128),
          // the rest waits below.
          if (C::RES) {
            if (it > 0 && item_of(it) / nMB != item_of(it - 1) / nMB) {
              umma_commit(bar_we);  // resident weights of the previous group no longer read
              ++epoch;
            }
            if (it == 0 || item_of(it) / nMB != item_of(it - 1) / nMB) mbar_wait(bar_wf, epoch & 1, sAbort);
          }
          mbar_wait(bar_p, it & 1, sAbort);
          tc_fence_after();
          for (int j = 0; j < nsub; ++j, ++c) {
            const int b = c & 1;
            if (j == 1 && it > 0) mbar_wait(bar_epd, (it - 1) & 1, sAbort);
            if (!C::RES) mbar_wait(bar_wf + c % C::D_NST, (c / C::D_NST) & 1, sAbort);
            tc_fence_after();
            if (!*sAbort) {
              const uint32_t aSt = s0 + C::D_W + (C::RES ? sub_of(j) : c % C::D_NST) * C::A_BYTES;
              const uint32_t tb = b * C::T_BUF3;
              kmma(tb, aPu, BM, 0, aSt, SC, 0, D / 16, ID_N, false);
              kmma(tb + SC, aPv, BM, 0, aSt + C::SUB_BYTES, SC, 0, D / 16, ID_N, false);
              kmma(tb + 2 * SC, aDY, BM, 0, aSt + 2 * C::SUB_BYTES, SC, 0, D / 16, ID_N, false);
            }
            umma_commit(bar_a + b);
            if (j == nsub - 1) umma_commit(bar_pf);
            if (j > 0) dp(c - 1);
          }
        }
        if (total > 0) dp(total - 1);
      } else if (role == R_UV) {
        auto products = [&](int it) {  // dB_u^T[h] += dU_h^T P_u, dB_v^T[h] += dV_h^T P_v
          const int x = (it + 1) * nsub - 1;
          mbar_wait(bar_du + (x & 1), (x >> 1) & 1, sAbort);
          tc_fence_after();
          if (!*sAbort) {
            const uint32_t aP = s0 + (it % NB_UV) * 3 * C::P_BYTES, aS = s0 + C::U_S;
            mnmma(C::T_ACCU, aS, aP, it > 0);
            mnmma(C::T_ACCV, aS + 2 * C::Z_BYTES, aP + C::P_BYTES, it > 0);
          }
          umma_commit(bar_w);
        };
        int c = 0;
        for (int it = 0; it < nit; ++it) {
          mbar_wait(bar_p + it % NB_UV, (it / NB_UV) & 1, sAbort);
          tc_fence_after();
          const uint32_t aP = s0 + (it % NB_UV) * 3 * C::P_BYTES;
          if (C::RES && it == 0) mbar_wait(bar_wf, 0, sAbort);
          for (int j = 0; j < nsub; ++j, ++c) {
            const int b = c & 1;
            if (c >= 2) mbar_wait(bar_du + b, ((c - 2) >> 1) & 1, sAbort);  // TMEM buffer b read out
            if (!C::RES) mbar_wait(bar_wf + b, (c >> 1) & 1, sAbort);
            tc_fence_after();
            if (!*sAbort) {
              const uint32_t aSt = s0 + C::U_W + (C::RES ? sub_of(j) : b) * C::A_BYTES;
              const uint32_t tb = b * C::T_BUF3;
              kmma(tb, aP, BM, 0, aSt, SC, 0, D / 16, ID_N, false);
              kmma(tb + SC, aP + C::P_BYTES, BM, 0, aSt + C::SUB_BYTES, SC, 0, D / 16, ID_N, false);
              kmma(tb + 2 * SC, aP + 2 * C::P_BYTES, BM, 0, aSt + 2 * C::SUB_BYTES, SC, 0, D / 16, ID_N, false);
            }
            umma_commit(bar_a + b);
            if (NB_UV == 2 && j == 0 && it > 0) products(it - 1);
          }
          if (NB_UV == 1) products(it);
        }
        if (NB_UV == 2 && nit > 0) products(nit - 1);
      } else {
        const uint32_t aPu = s0 + C::OFF_PU, aPv = s0 + C::OFF_PV, aH = s0 + C::OFF_X1, aZP = s0 + C::O_ZP;
        constexpr int SPP = 128 / SC;  // sub-chunks per 128-feature pair
        auto y = [&](int x) {  // Y += Z_x B_o[x]; M_o[pair] += Z_pair^T H once a pair is complete
          const int bx = x & 1, jx = x % nsub, itx = x / nsub, kx = x / C::SPC;
          mbar_wait(bar_du + bx, (x >> 1) & 1, sAbort);  // Z_x in the pair buffer
          if (!C::RES && x % C::SPC == 0) mbar_wait(bar_bo + (kx & 1), (kx >> 1) & 1, sAbort);
          tc_fence_after();
          if (!*sAbort) {
            const uint32_t aBo = s0 + C::O_BO + (C::RES ? sub_of(jx) / C::SPC : kx & 1) * C::BO_BYTES;
            kmma(C::T_Y, aZP, BM, (jx % SPP) * (SC / 16), aBo, D, (x % C::SPC) * (SC / 16), SC / 16, ID_ND, jx > 0);
          }
          if (!C::RES && x % C::SPC == C::SPC - 1) umma_commit(bar_boe + (kx & 1));
          if (jx == nsub - 1) umma_commit(bar_yd);
          if (jx % SPP == SPP - 1) {
            if (jx == SPP - 1) {
              mbar_wait(bar_gl, itx & 1, sAbort);  // H of this item
              tc_fence_after();
            }
            if (!*sAbort) mnmma(C::T_ACCO + (sub_of(jx) / SPP) * D, aZP, aH, itx > 0);
            umma_commit(bar_w);
          }
        };
        int c = 0;
        for (int it = 0; it < nit; ++it) {
          if (c > 0) y(c - 1);  // finish the previous item before waiting for this one's operands
          // The epilogue's warp-level MMAs share the tensor pipe: only this
          // item's first U/V go ahead of them (the compute warps find them done
          // when the epilogue ends; the epilogue's closing barrier orders the
          // reuse of the Z pair buffer), the rest waits below.
          if (C::RES && it == 0) mbar_wait(bar_wf, 0, sAbort);
          mbar_wait(bar_p, it & 1, sAbort);
          tc_fence_after();
          for (int j = 0; j < nsub; ++j, ++c) {
            const int b = c & 1;
            if (j == 1 && it > 0) mbar_wait(bar_epd, (it - 1) & 1, sAbort);
            if (!C::RES) mbar_wait(bar_wf + b, (c >> 1) & 1, sAbort);
            tc_fence_after();
            if (!*sAbort) {
              const uint32_t aSt = s0 + C::O_W1 + (C::RES ? sub_of(j) : b) * 2 * C::SUB_BYTES;
              const uint32_t tb = b * C::T_BUF2;
              kmma(tb, aPu, BM, 0, aSt, SC, 0, D / 16, ID_N, false);
              kmma(tb + SC, aPv, BM, 0, aSt + C::SUB_BYTES, SC, 0, D / 16, ID_N, false);
            }
            umma_commit(bar_a + b);
            if (j == nsub - 1) umma_commit(bar_pf);
            if (j > 0) y(c - 1);
          }
        }
        if (total > 0) y(total - 1);
      }
    }
  } else {
    // ------------------------------------------------ compute warps
    const int tid = threadIdx.x;
    const int g = lane >> 2, t4 = lane & 3;
    const int lq = warp & 3, chh = warp >> 2;
    const int r = lq * 32 + lane;
    const uint32_t trow = tbase + ((uint32_t)(lq * 32) << 16);
    const int cb = chh * HC;
    auto frag = [&](int m, bool tr, uint32_t (&f)[4]) { load_afrag(a.amat + m * 256, tr, g, t4, f); };
    float accA[2][2][4] = {};  // DGRAD: dA_u, dA_v ; O: dA_o in accA[0]
    int c = 0, pc = 0;
    // DGRAD epilogue metadata, loaded into registers one item ahead.  The
    // loads are unconditional (clamped index) and their values are first used
    // where the metadata is stored, so issuing them does not wait for memory.
    struct MetaReg { int tok, b, ch, cont; bool valid; };
    auto meta_issue = [&](int it) {
      MetaReg m{0, 0, 0, 0, false};
      const int64_t item = item_of(it);
      const int qc = (int)(item / nMB), mb = (int)(item - (int64_t)qc * nMB);
      if (tid < BM) {
        const int64_t t = (int64_t)mb * 8 + (tid >> 4);
        m.valid = t < BQ;
        const int64_t tc = m.valid ? t : 0;
        // 32-bit division whenever the tile count allows (it always does at
        // the supported batch sizes); the 64-bit one costs ~1000 cycles.
        m.b = BQ < (int64_t)INT32_MAX ? (int)tc / p.Qs : (int)(tc / p.Qs);
        m.tok = p.tok[(tc - (int64_t)m.b * p.Qs) * 16 + (tid & 15)];
      }
      if (tid < D) m.ch = p.ch[qc * D + tid];
      if (tid == 0) m.cont = a.contig[qc];
      return m;
    };
    MetaReg mreg{0, 0, 0, 0, false};
    if (role == R_DGRAD && nit > 0) mreg = meta_issue(0);
    for (int it = 0; it < nit; ++it) {
      const int64_t item = item_of(it);
      const int qc = (int)(item / nMB);
      const float* ggq = a.gg + (int64_t)qc * D;

      // ---- sub-chunk loop
      for (int j = 0; j < nsub; ++j, ++c) {
        const int b = c & 1;
        mbar_wait(bar_a + b, (c >> 1) & 1, sAbort);
        __syncwarp();
        tc_fence_after();
        if (role != R_O) {
          uint32_t ur[HC], vr[HC], zr[HC];
          const uint32_t tcol = b * C::T_BUF3 + cb;
          tmem_ld_cols<HC>(trow + tcol, ur);
          tmem_ld_cols<HC>(trow + tcol + SC, vr);
          tmem_ld_cols<HC>(trow + tcol + 2 * SC, zr);
          tmem_ld_wait();
          // The math runs before the wait for the destination buffer, so it
          // overlaps the MMAs still reading that buffer (DGRAD: dP of
          // sub-chunk c - 2; UV: the previous item's weight-gradient products).
          uint32_t wu[HC / 8][4], wv[HC / 8][4];
#pragma unroll
          for (int jj = 0; jj < HC / 8; ++jj) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              // Two features at a time in packed f32x2 arithmetic:
              // s = sigmoid(u), dV = dZ s u, dU = dZ s v (1 + u (1 - s)).
              const int i = jj * 8 + 2 * e;
              const uint64_t u2 = f2pack(__uint_as_float(ur[i]), __uint_as_float(ur[i + 1]));
              const uint64_t v2 = f2pack(__uint_as_float(vr[i]), __uint_as_float(vr[i + 1]));
              const uint64_t z2 = f2pack(__uint_as_float(zr[i]), __uint_as_float(zr[i + 1]));
              const uint64_t half = f2pack(0.5f, 0.5f), nhalf = f2pack(-0.5f, -0.5f), one = f2pack(1.f, 1.f);
              const float2 h = f2unpack(mul2(u2, half));
              float t0, t1;
              asm("tanh.approx.f32 %0, %1;" : "=f"(t0) : "f"(h.x));
              asm("tanh.approx.f32 %0, %1;" : "=f"(t1) : "f"(h.y));
              const uint64_t t2 = f2pack(t0, t1);
              const uint64_t s2 = fma2(t2, half, half);      // sigmoid(u)
              const uint64_t oms = fma2(t2, nhalf, half);    // 1 - sigmoid(u)
              const uint64_t ds2 = mul2(z2, s2);
              const float2 dv = f2unpack(mul2(ds2, u2));
              const float2 du = f2unpack(mul2(mul2(ds2, v2), fma2(u2, oms, one)));
              wu[jj][e] = pack2<BF16>(du.x, du.y);
              wv[jj][e] = pack2<BF16>(dv.x, dv.y);
            }
          }
          unsigned char* du_at;
          int col0;
          int dv_off;
          if (role == R_DGRAD) {
            if (c >= 2) mbar_wait(bar_b + b, ((c - 2) >> 1) & 1, sAbort);  // dP(c-2) read this buffer
            du_at = sm + C::D_S + buf_atom(b, 2);
            dv_off = C::Z_BYTES;
            col0 = buf_col(b);
          } else {
            if (j == 0 && it > 0) mbar_wait(bar_w, (it - 1) & 1, sAbort);  // products read dU_h / dV_h
            du_at = sm + C::U_S;
            dv_off = 2 * C::Z_BYTES;
            col0 = sub_of(j) * SC;
          }
#pragma unroll
          for (int jj = 0; jj < HC / 8; ++jj) {
            const uint32_t off = sw128_off(r, col0 + cb + jj * 8, BM);
            *reinterpret_cast<uint4*>(du_at + off) = make_uint4(wu[jj][0], wu[jj][1], wu[jj][2], wu[jj][3]);
            *reinterpret_cast<uint4*>(du_at + dv_off + off) = make_uint4(wv[jj][0], wv[jj][1], wv[jj][2], wv[jj][3]);
          }
        } else {  // R_O: Z = silu(U) * V into the pair buffer at feature offset fo
          uint32_t ur[HC], vr[HC];
          const uint32_t tcol = b * C::T_BUF2 + cb;
          tmem_ld_cols<HC>(trow + tcol, ur);
          tmem_ld_cols<HC>(trow + tcol + SC, vr);
          tmem_ld_wait();
          const int fo = (j % (128 / SC)) * SC;
          uint32_t wz[HC / 8][4];
#pragma unroll
          for (int jj = 0; jj < HC / 8; ++jj) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int i0 = jj * 8 + 2 * e;
              const uint32_t u2 = pack2<BF16>(__uint_as_float(ur[i0]), __uint_as_float(ur[i0 + 1]));
              const uint32_t v2 = pack2<BF16>(__uint_as_float(vr[i0]), __uint_as_float(vr[i0 + 1]));
              wz[jj][e] = silu_mul2<BF16>(u2, v2);
            }
          }
          // The previous pair's M_o (issued after its Y MMAs) has read the buffer.
          if (fo == 0 && pc > 0) mbar_wait(bar_w, (pc - 1) & 1, sAbort);
          unsigned char* sz = sm + C::O_ZP;
#pragma unroll
          for (int jj = 0; jj < HC / 8; ++jj)
            *reinterpret_cast<uint4*>(sz + sw128_off(r, fo + cb + jj * 8, BM)) =
                make_uint4(wz[jj][0], wz[jj][1], wz[jj][2], wz[jj][3]);
          if (fo + SC == 128) ++pc;
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(bar_du + b);
      }

      // ---- per-item epilogue
      if (role == R_DGRAD) {
        // Metadata of this item for the dX scatter.
        if (tid < BM) sRow[tid] = mreg.valid && mreg.tok < p.N ? mreg.b * p.N + mreg.tok : -1;
        if (tid < D) sCh[tid] = mreg.ch;
        if (tid == 0) *sCont = a.vec_ok ? mreg.cont : 0;
        comp_sync();
        if (it + 1 < nit) mreg = meta_issue(it + 1);
        const int lay = *sCont;
        const bool cont = layout_stride(lay) == 1;
        const int sstride = layout_stride(lay) > 1 ? layout_stride(lay) : 0, sc0 = layout_c0(lay);
        mbar_wait(bar_b + ((c - 1) & 1), ((c - 1) >> 1) & 1, sAbort);  // last dP of the item done
        __syncwarp();
        tc_fence_after();
        // Warp (lq, hw): tiles 2lq, 2lq+1 (TMEM lanes 32lq..32lq+31), channels
        // [hw*D/2, (hw+1)*D/2).  dP arrives in the mma C-fragment layout.
        constexpr int NP = D / 32;
        const int hw = warp >> 2;
        // Pass 1: dT = A_u^T dP_u + A_v^T dP_v -> dX (needs no T).  Warp
        // (lq, hw) owns tile 2 lq + hw and all D channels.  Per 64-channel pass
        // each half-tile (rows g / g + 8 of the C fragments) goes through the
        // warp's f32 staging tile, so that 16 lanes write one row segment.
        {
          uint32_t fuT[4], fvT[4];
          frag(0, true, fuT);
          frag(1, true, fvT);
          const int tile = 2 * lq + hw;
          const int rwA = sRow[tile * 16 + g], rwB = sRow[tile * 16 + g + 8];
          const uint32_t tl_addr = tbase + ((uint32_t)(tile * 16) << 16);
          float* stg = reinterpret_cast<float*>(sm + C::D_STG + warp * C::D_STG_WARP);
#pragma unroll 1
          for (int hf = 0; hf < D / 64; ++hf) {
            uint32_t pu[4][8], pv[4][8];
#pragma unroll
            for (int n4 = 0; n4 < 4; ++n4) {
              const int k0 = hf * 64 + n4 * 16;
              tmem_ld16x256_x2(tl_addr + C::T_DPU + k0, pu[n4]);
              tmem_ld16x256_x2(tl_addr + C::T_DPV + k0, pv[n4]);
            }
            tmem_ld_wait();
            float cc[4][2][4];  // [16-channel step][channel block nb][C fragment]
#pragma unroll
            for (int n4 = 0; n4 < 4; ++n4) {
              uint32_t au[4], av[4];
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                au[q] = pack2<BF16>(__uint_as_float(pu[n4][2 * q]), __uint_as_float(pu[n4][2 * q + 1]));
                av[q] = pack2<BF16>(__uint_as_float(pv[n4][2 * q]), __uint_as_float(pv[n4][2 * q + 1]));
              }
#pragma unroll
              for (int nb = 0; nb < 2; ++nb) {
                cc[n4][nb][0] = cc[n4][nb][1] = cc[n4][nb][2] = cc[n4][nb][3] = 0.f;
                const uint32_t bu0 = movm_trans(au[2 * nb]), bu1 = movm_trans(au[2 * nb + 1]);
                const uint32_t bv0 = movm_trans(av[2 * nb]), bv1 = movm_trans(av[2 * nb + 1]);
                mma16816<BF16>(cc[n4][nb], fuT, bu0, bu1);
                mma16816<BF16>(cc[n4][nb], fvT, bv0, bv1);
              }
            }
            if (sstride) {
              // Strided group (channels sc0 + S k): the half-tile goes through
              // the staging tile too; 16 lanes then store 16 consecutive k of
              // one row, which lie S elements apart in dX.
#pragma unroll
              for (int hr = 0; hr < 2; ++hr) {
#pragma unroll
                for (int n4 = 0; n4 < 4; ++n4)
#pragma unroll
                  for (int nb = 0; nb < 2; ++nb)
                    *reinterpret_cast<float2*>(stg + g * C::D_ST_LD + n4 * 16 + nb * 8 + 2 * t4) =
                        make_float2(cc[n4][nb][2 * hr], cc[n4][nb][2 * hr + 1]);
                __syncwarp();
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  const int r8 = (i * 32 + lane) >> 4;
                  const int rw = sRow[tile * 16 + hr * 8 + r8];
                  if (rw >= 0) {
                    const int64_t rowoff = (int64_t)rw * p.C + sc0 + (int64_t)sstride * hf * 64;
#pragma unroll
                    for (int m = 0; m < 4; ++m) {
                      const int k = (lane & 15) + 16 * m;
                      const float v = stg[r8 * C::D_ST_LD + k];
                      const int64_t off = rowoff + (int64_t)sstride * k;
                      if (a.dxn) reinterpret_cast<T16*>(a.dxn)[off] = Elem<T16>::from(v);
                      else ((TX*)a.dx)[off] = Elem<TX>::from(v);
                    }
                  }
                }
                __syncwarp();  // the staging tile is rewritten by the next half-tile
              }
            } else if (cont) {
#pragma unroll
              for (int hr = 0; hr < 2; ++hr) {
#pragma unroll
                for (int n4 = 0; n4 < 4; ++n4)
#pragma unroll
                  for (int nb = 0; nb < 2; ++nb)
                    *reinterpret_cast<float2*>(stg + g * C::D_ST_LD + n4 * 16 + nb * 8 + 2 * t4) =
                        make_float2(cc[n4][nb][2 * hr], cc[n4][nb][2 * hr + 1]);
                __syncwarp();
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  const int r8 = (i * 32 + lane) >> 4, c4 = (lane & 15) * 4;
                  const float4 v = *reinterpret_cast<const float4*>(stg + r8 * C::D_ST_LD + c4);
                  const int rw = sRow[tile * 16 + hr * 8 + r8];
                  if (rw >= 0) {
                    const int64_t off = (int64_t)rw * p.C + sCh[0] + hf * 64 + c4;
                    if (a.dxn) {
                      *reinterpret_cast<uint2*>(reinterpret_cast<T16*>(a.dxn) + off) =
                          make_uint2(pack2<BF16>(v.x, v.y), pack2<BF16>(v.z, v.w));
                    } else if constexpr (std::is_same_v<TX, float>) {
                      *reinterpret_cast<float4*>((float*)a.dx + off) = v;
                    } else {
                      constexpr bool XB = std::is_same_v<TX, __nv_bfloat16>;
                      *reinterpret_cast<uint2*>((TX*)a.dx + off) = make_uint2(pack2<XB>(v.x, v.y), pack2<XB>(v.z, v.w));
                    }
                  }
                }
                __syncwarp();  // the staging tile is rewritten by the next half-tile
              }
            } else {
#pragma unroll
              for (int n4 = 0; n4 < 4; ++n4)
#pragma unroll
                for (int nb = 0; nb < 2; ++nb) {
                  const int k = hf * 64 + n4 * 16 + nb * 8 + 2 * t4;
#pragma unroll
                  for (int hr = 0; hr < 2; ++hr) {
                    const int rw = hr ? rwB : rwA;
                    if (rw < 0) continue;
                    const int64_t row = rw;
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                      const int ch = sCh[k + e];
                      if (ch >= p.C) continue;
                      const int64_t off = row * p.C + ch;
                      const float dv = cc[n4][nb][2 * hr + e];
                      if (a.dxn) reinterpret_cast<T16*>(a.dxn)[off] = Elem<T16>::from(dv);
                      else ((TX*)a.dx)[off] = Elem<TX>::from(dv);
                    }
                  }
                }
            }
          }
        }
        // Pass 2: dA_u += dP_u T^T, dA_v += dP_v T^T with T from its image.
        mbar_wait(bar_t, it & 1, sAbort);
        __syncwarp();
        {
          const uint32_t aT = smem_u32(sm + C::D_TT);
#pragma unroll 1
          for (int tl = 0; tl < 2; ++tl) {
            const int tile = 2 * lq + tl;
            const uint32_t tl_addr = tbase + ((uint32_t)(tile * 16) << 16);
            uint32_t pu[NP][8], pv[NP][8];
#pragma unroll
            for (int np = 0; np < NP; ++np) {
              const int k0 = hw * (D / 2) + np * 16;
              tmem_ld16x256_x2(tl_addr + C::T_DPU + k0, pu[np]);
              tmem_ld16x256_x2(tl_addr + C::T_DPV + k0, pv[np]);
            }
            tmem_ld_wait();
#pragma unroll
            for (int np = 0; np < NP; ++np) {
              const int k0 = hw * (D / 2) + np * 16;
              uint32_t au[4], av[4];
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                au[q] = pack2<BF16>(__uint_as_float(pu[np][2 * q]), __uint_as_float(pu[np][2 * q + 1]));
                av[q] = pack2<BF16>(__uint_as_float(pv[np][2 * q]), __uint_as_float(pv[np][2 * q + 1]));
              }
              // B[k = channel][n = token j] = T[j][k]
              uint32_t tb[4];
              ldsm_x4(aT + sw128_off(tile * 16 + (lane & 7) + (lane >> 4) * 8, k0 + ((lane >> 3) & 1) * 8, BM),
                      tb[0], tb[1], tb[2], tb[3]);
              mma16816<BF16>(accA[0][0], au, tb[0], tb[1]);
              mma16816<BF16>(accA[0][1], au, tb[2], tb[3]);
              mma16816<BF16>(accA[1][0], av, tb[0], tb[1]);
              mma16816<BF16>(accA[1][1], av, tb[2], tb[3]);
            }
          }
        }
        tc_fence_before();
        mbar_arrive(bar_epd);  // T region free for the next item's T
        comp_sync();  // T and the metadata are read out
      } else if (role == R_O) {
        mbar_wait(bar_yd, it & 1, sAbort);        // Y complete
        mbar_wait(bar_w, (pc - 1) & 1, sAbort);   // last M_o done with the pair buffer
        mbar_wait(bar_gl, it & 1, sAbort);        // H and G' of this item present
        __syncwarp();
        tc_fence_after();
        unsigned char* stY = sm + C::O_ZP;
        const uint32_t aY = smem_u32(stY), aG = smem_u32(sm + C::O_G);
        const int cb32 = chh * 32;
        for (int hf = 0; hf < D / 64; ++hf) {
          uint32_t yr[32];
          tmem_ld32(trow + C::T_Y + hf * 64 + cb32, yr);
          tmem_ld_wait();
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            uint4 w;
            const int k = hf * 64 + cb32 + jj * 8;
            w.x = pack2<BF16>(__uint_as_float(yr[jj * 8 + 0]) * ggq[k + 0], __uint_as_float(yr[jj * 8 + 1]) * ggq[k + 1]);
            w.y = pack2<BF16>(__uint_as_float(yr[jj * 8 + 2]) * ggq[k + 2], __uint_as_float(yr[jj * 8 + 3]) * ggq[k + 3]);
            w.z = pack2<BF16>(__uint_as_float(yr[jj * 8 + 4]) * ggq[k + 4], __uint_as_float(yr[jj * 8 + 5]) * ggq[k + 5]);
            w.w = pack2<BF16>(__uint_as_float(yr[jj * 8 + 6]) * ggq[k + 6], __uint_as_float(yr[jj * 8 + 7]) * ggq[k + 7]);
            *reinterpret_cast<uint4*>(stY + (r * STG_LD + cb32 + jj * 8) * 2) = w;
          }
          comp_sync();
          __syncwarp();
          auto rowG = [&](int rr, int k) { return aG + sw128_off(warp * 16 + rr, hf * 64 + k, BM); };
          auto rowY = [&](int rr, int k) { return aY + ((warp * 16 + rr) * STG_LD + k) * 2; };
          gram16<BF16>(accA[0], rowG, rowY, lane);
          comp_sync();
        }
        tc_fence_before();
        mbar_arrive(bar_epd);
      }
    }

    // ---- end of the CTA's items: write partials
    if (role == R_DGRAD) {
      float* dst = a.pdA + ((int64_t)blockIdx.x * NCOMP_WARPS + warp) * 512;
#pragma unroll
      for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int nb = 0; nb < 2; ++nb) {
          const int col = nb * 8 + 2 * t4;
          dst[m * 256 + g * 16 + col] = accA[m][nb][0];
          dst[m * 256 + g * 16 + col + 1] = accA[m][nb][1];
          dst[m * 256 + (g + 8) * 16 + col] = accA[m][nb][2];
          dst[m * 256 + (g + 8) * 16 + col + 1] = accA[m][nb][3];
        }
    } else if (n_items > 0) {
      if (role == R_UV) mbar_wait(bar_w, (nit - 1) & 1, sAbort);
      else mbar_wait(bar_w, (pc - 1) & 1, sAbort);
      __syncwarp();
      tc_fence_after();
      const int cb32 = chh * 32;
      if (role == R_UV) {
        float* dst = a.puv + (int64_t)wslot * 2 * 128 * D;
        for (int m = 0; m < 2; ++m)
          for (int c0 = 0; c0 < D; c0 += 64) {
            uint32_t vr[32];
            tmem_ld32(trow + (m ? C::T_ACCV : C::T_ACCU) + c0 + cb32, vr);
            tmem_ld_wait();
            float* o = dst + ((int64_t)m * 128 + r) * D + c0 + cb32;
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              *reinterpret_cast<float4*>(o + i) = make_float4(__uint_as_float(vr[i]), __uint_as_float(vr[i + 1]),
                                                              __uint_as_float(vr[i + 2]), __uint_as_float(vr[i + 3]));
          }
      } else {
        float* dst = a.po + (int64_t)wslot * C::RD * D;
        for (int hb = 0; hb < C::NH; ++hb)
          for (int c0 = 0; c0 < D; c0 += 64) {
            uint32_t vr[32];
            tmem_ld32(trow + C::T_ACCO + hb * D + c0 + cb32, vr);
            tmem_ld_wait();
            float* o = dst + ((int64_t)hb * 128 + r) * D + c0 + cb32;
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              *reinterpret_cast<float4*>(o + i) = make_float4(__uint_as_float(vr[i]), __uint_as_float(vr[i + 1]),
                                                              __uint_as_float(vr[i + 2]), __uint_as_float(vr[i + 3]));
          }
        float* da = a.pdAo + ((int64_t)wslot * NCOMP_WARPS + warp) * 256;
#pragma unroll
        for (int nb = 0; nb < 2; ++nb) {
          const int col = nb * 8 + 2 * t4;
          da[g * 16 + col] = accA[0][nb][0];
          da[g * 16 + col + 1] = accA[0][nb][1];
          da[(g + 8) * 16 + col] = accA[0][nb][2];
          da[(g + 8) * 16 + col + 1] = accA[0][nb][3];
        }
      }
      tc_fence_before();
    } else if (role == R_O) {
      float* da = a.pdAo + ((int64_t)wslot * NCOMP_WARPS + warp) * 256;
      for (int i = lane; i < 256; i += 32) da[i] = 0.f;
      float* dst = a.po + (int64_t)wslot * C::RD * D;
      for (int i = tid; i < C::RD * D; i += NCOMP) dst[i] = 0.f;
    } else {
      float* dst = a.puv + (int64_t)wslot * 2 * 128 * D;
      for (int i = tid; i < 2 * 128 * D; i += NCOMP) dst[i] = 0.f;
    }
  }

  __syncwarp();
  __syncthreads();
  report_abort(sAbort, a.fault);
  if (*sAbort) {
    for (int i = 0; i < 1000; ++i) __nanosleep(1000);
  }
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tbase, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Reduction of the per-CTA partials into the gradient outputs.  Every sum is
// taken in a fixed order (per-thread loops over partial slots, then a fixed
// shuffle tree), so results are bitwise reproducible.
// ---------------------------------------------------------------------------
// dB_u, dB_v [qc][c][e] and M_o -> dB_o [qc][e][c]: one thread per output,
// consecutive threads on consecutive c so the partial reads coalesce.
// Sum of at(0) + at(1) + ... + at(n - 1) in that order (bitwise reproducible),
// with the loads requested eight at a time so their latencies overlap.
template <typename F>
__device__ __forceinline__ float sum_in_order(int64_t n, F at) {
  float s = 0.f;
  for (int64_t j = 0; j < n; j += 8) {
    float v[8];
    // Unconditional loads from a clamped index; only the first n terms count.
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = at(j + k < n ? j + k : n - 1);
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (j + k < n) s += v[k];
  }
  return s;
}

template <int D, typename TW>
__global__ void tc_bwd_reduce_b_kernel(Prob p, BwdArgs a, TW* __restrict__ db_u, TW* __restrict__ db_v,
                                       TW* __restrict__ db_o, float* __restrict__ mo) {
  using C = BCfg<D>;
  const int tid = blockIdx.x * blockDim.x + threadIdx.x;
  const int stride = gridDim.x * blockDim.x;
  const int nB = p.Qc * D * C::RD;
  for (int i = tid; i < 3 * nB; i += stride) {
    const int m = i / nB;
    const int rem = i - m * nB;
    const int qc = rem / (C::RD * D);
    const int e = (rem / D) % C::RD, c = rem % D;
    if (m < 2) {
      const int hh = e / 128, el = e % 128;
      const float* src = a.puv + ((((int64_t)(hh * p.Qc + qc) * a.nUVq) * 2 + m) * 128 + el) * D + c;
      const int64_t st = (int64_t)2 * 128 * D;
      const float s = sum_in_order(a.nUVq, [&](int64_t j) { return __ldg(src + j * st); });
      (m ? db_v : db_u)[((int64_t)qc * D + c) * C::RD + e] = Elem<TW>::from(s);
    } else {
      const float* src = a.po + (int64_t)qc * a.nOq * C::RD * D + (int64_t)e * D + c;
      const float s = sum_in_order(a.nOq, [&](int64_t j) { return __ldg(src + j * (int64_t)C::RD * D); });
      mo[rem] = s;
      db_o[rem] = Elem<TW>::from(s * a.gg[(int64_t)qc * D + c]);
    }
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// dgamma[ch[qc][c]] = sum_e B_o[qc][e][c] * M_o[qc][e][c]  (one warp per (qc, c)),
// and the token-mix gradients (one warp per element).
template <int D, typename TW>
__global__ void tc_bwd_reduce_small_kernel(Prob p, BwdArgs a, const TW* __restrict__ bo,
                                           const float* __restrict__ mo, TW* __restrict__ dgamma,
                                           TW* __restrict__ da_u, TW* __restrict__ da_v, TW* __restrict__ da_o) {
  using C = BCfg<D>;
  const int lane = threadIdx.x & 31;
  const int64_t gw = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t n_gamma = (int64_t)p.Qc * D;
  for (int64_t w = gw; w < n_gamma + 3 * 256; w += nw) {
    float s = 0.f;
    if (w < n_gamma) {
      const int qc = (int)(w / D), c = (int)(w % D);
      float bv[C::RD / 32], mv[C::RD / 32];
#pragma unroll
      for (int k = 0; k < C::RD / 32; ++k) {
        const int64_t idx = ((int64_t)qc * C::RD + lane + 32 * k) * D + c;
        bv[k] = load_as<float>(bo, idx);
        mv[k] = mo[idx];
      }
#pragma unroll
      for (int k = 0; k < C::RD / 32; ++k) s += bv[k] * mv[k];
      s = warp_sum(s);
      const int ch = p.ch[w];
      if (lane == 0 && ch < p.C) dgamma[ch] = Elem<TW>::from(s);
    } else {
      const int m = (int)((w - n_gamma) / 256), e = (int)((w - n_gamma) % 256);
      // Lane l sums partials l, l + 32, ... in order, then a fixed butterfly.
      if (m < 2) {
        const int64_t n = (int64_t)a.nD * NCOMP_WARPS;
        const float* src = a.pdA + (int64_t)lane * 512 + m * 256 + e;
        s = sum_in_order(n > lane ? (n - 1 - lane) / 32 + 1 : 0, [&](int64_t k) { return __ldg(src + k * 32 * 512); });
      } else {
        const int64_t n = (int64_t)p.Qc * a.nOq * NCOMP_WARPS;
        const float* src = a.pdAo + (int64_t)lane * 256 + e;
        s = sum_in_order(n > lane ? (n - 1 - lane) / 32 + 1 : 0, [&](int64_t k) { return __ldg(src + k * 32 * 256); });
      }
      s = warp_sum(s);
      if (lane == 0) (m == 0 ? da_u : (m == 1 ? da_v : da_o))[e] = Elem<TW>::from(s);
    }
  }
}

template <int D, bool BF16>
int tc_backward_t(const ow_bigemm_args_t* ar, const ow_bigemm_grads_t* gr, const Prob& p, cudaStream_t st,
                  Carver& ws) {
  const bool block = ar->rstd != nullptr;
  BPlan<D> pl(p, block, device_sm_count());
  unsigned char* base = (unsigned char*)ws.take(pl.total);
  NormBwd nbw{};
  if (block) nbw = norm_bwd_take((int64_t)p.B * p.N, p.C, ws);
  if (!ws.base) return OW_OK;
  BwdArgs a{};
  OW_RETURN_IF(fault_word(&a.fault));
  a.probe_ns = wait_probe_ns();
  a.p = p;
  a.x = ar->x;
  a.dout = gr->dout;
  a.rstd = (const float*)ar->rstd;
  a.scale = ar->sample_scale;
  a.x_dt = ar->x_dtype;
  a.img = base + pl.img;
  a.amat = (const uint16_t*)(base + pl.amat);
  a.gg = (const float*)(base + pl.gg);
  a.nw = (const float*)(base + pl.nw);
  a.contig = (const int*)(base + pl.contig);
  a.vec_ok = ((uintptr_t)ar->x % 16 == 0) && ((uintptr_t)gr->dout % 16 == 0) && ((uintptr_t)gr->dx % 16 == 0) &&
             (p.C % 8 == 0);
  a.dx = block ? nullptr : gr->dx;
  a.dxn = block ? (void*)(base + pl.dxn) : nullptr;
  a.pdA = (float*)(base + pl.pdA);
  a.pdAo = (float*)(base + pl.pdAo);
  a.puv = (float*)(base + pl.puv);
  a.po = (float*)(base + pl.po);
  a.packed = base + pl.packed;
  a.nD = pl.nD;
  a.nUVq = pl.nUVq;
  a.nOq = pl.nOq;
  a.nH = pl.nH;

  // Weight images.
  {
    const int64_t n = 4LL * p.Qc * 2 * D * D;
    const int grid = (int)std::min<int64_t>((n + 255) / 256, 148 * 8);
    auto run = [&](auto* tw) {
      using TW = std::remove_pointer_t<decltype(tw)>;
      launch(tc_bwd_prep_kernel<D, TW, BF16>, grid, 256, 0, st, p, (const TW*)ar->a_u, (const TW*)ar->a_v,
             (const TW*)ar->a_o, (const TW*)ar->b_u, (const TW*)ar->b_v, (const TW*)ar->b_o,
             (const TW*)ar->gamma, (const TW*)(block ? ar->norm_w : nullptr), base + pl.img,
             (uint16_t*)(base + pl.amat), (float*)(base + pl.gg), (float*)(base + pl.nw),
             (int*)(base + pl.contig));
    };
    switch (ar->w_dtype) {
      case OW_DTYPE_F32: run((float*)nullptr); break;
      case OW_DTYPE_F64: run((double*)nullptr); break;
      case OW_DTYPE_BF16: run((__nv_bfloat16*)nullptr); break;
      case OW_DTYPE_F16: run((__half*)nullptr); break;
      default: set_error("unsupported weight dtype"); return OW_ERR_UNSUPPORTED;
    }
    OW_CHECK_LAUNCH("tc_bwd_prep_kernel");
  }

  auto go = [&](auto* tx, auto* to) -> int {
    using TX = std::remove_pointer_t<decltype(tx)>;
    using TO = std::remove_pointer_t<decltype(to)>;
    const int64_t items = (int64_t)p.Qc * ((p.BQ() + 7) / 8);
    if (items > 0) {
      constexpr int pack_smem = 3 * BM * 128 + STG_BYTES + (BM + D) * 4 + 128;
      auto pk = tc_pack_kernel<D, BF16, TX, TO>;
      cudaError_t pe = cudaFuncSetAttribute(pk, cudaFuncAttributeMaxDynamicSharedMemorySize, pack_smem);
      if (pe != cudaSuccess) {
        set_error("tc backward: cannot reserve %d bytes of shared memory for the pack kernel: %s", pack_smem,
                  cudaGetErrorString(pe));
        return OW_ERR_CUDA;
      }
      profile_mark(OW_PROF_PACK, false, st);
      launch(pk, (int)items, NCOMP, pack_smem, st, a);
      profile_mark(OW_PROF_PACK, true, st);
      OW_CHECK_LAUNCH("tc_pack_kernel");
    }
    auto kern = tc_bwd_kernel<D, BF16, TX, TO>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, BCfg<D>::SMEM);
    if (e != cudaSuccess) {
      set_error("tc backward: cannot reserve %d bytes of shared memory: %s", BCfg<D>::SMEM, cudaGetErrorString(e));
      return OW_ERR_CUDA;
    }
    profile_mark(OW_PROF_BWD, false, st);
    launch(kern, pl.grid, TC_THREADS, BCfg<D>::SMEM, st, a);
    profile_mark(OW_PROF_BWD, true, st);
    OW_CHECK_LAUNCH("tc_bwd_kernel");
    return OW_OK;
  };
  using T16 = std::conditional_t<BF16, __nv_bfloat16, __half>;
  const int xd = ar->x_dtype, od = ar->out_dtype;
  const int c16 = BF16 ? OW_DTYPE_BF16 : OW_DTYPE_F16;
  int rc;
  if (xd == c16 && od == c16) rc = go((T16*)nullptr, (T16*)nullptr);
  else if (xd == c16 && od == OW_DTYPE_F32) rc = go((T16*)nullptr, (float*)nullptr);
  else if (xd == OW_DTYPE_F32 && od == OW_DTYPE_F32) rc = go((float*)nullptr, (float*)nullptr);
  else if (xd == OW_DTYPE_F32 && od == c16) rc = go((float*)nullptr, (T16*)nullptr);
  else {
    set_error("tc backward: unsupported dtypes x=%s out=%s", dtype_name(xd), dtype_name(od));
    return OW_ERR_UNSUPPORTED;
  }
  OW_RETURN_IF(rc);

  auto red = [&](auto* tw) {
    using TW = std::remove_pointer_t<decltype(tw)>;
    float* mo = (float*)(base + pl.mo);
    launch(tc_bwd_reduce_b_kernel<D, TW>, (int)std::min<int64_t>((3LL * p.Qc * D * 2 * D + 255) / 256, 148 * 32), 256,
           0, st, p, a, (TW*)gr->db_u, (TW*)gr->db_v,
           (TW*)gr->db_o, mo);
    launch(tc_bwd_reduce_small_kernel<D, TW>, 148, 256, 0, st, p, a, (const TW*)ar->b_o, (const float*)mo,
           (TW*)gr->dgamma, (TW*)gr->da_u, (TW*)gr->da_v, (TW*)gr->da_o);
  };
  switch (ar->w_dtype) {
    case OW_DTYPE_F32: red((float*)nullptr); break;
    case OW_DTYPE_F64: red((double*)nullptr); break;
    case OW_DTYPE_BF16: red((__nv_bfloat16*)nullptr); break;
    case OW_DTYPE_F16: red((__half*)nullptr); break;
  }
  OW_CHECK_LAUNCH("tc_bwd_reduce_kernel");
  if (block)
    return norm_bwd_run(nbw, ar->x, ar->x_dtype, gr->dout, ar->out_dtype, (const float*)ar->rstd,
                        (const float*)(base + pl.nw), a.dxn, BF16 ? OW_DTYPE_BF16 : OW_DTYPE_F16,
                        (int64_t)p.B * p.N, p.C, gr->dx, gr->dnorm_w,
                        ar->w_dtype, st);
  return OW_OK;
}

}  // namespace

namespace {
template <int D, bool BF16>
int tc_pack_forward_t(const ow_bigemm_args_t* ar, const Prob& p, const uint16_t* amat, const float* nwc,
                      const int* contig, unsigned char* packed, cudaStream_t st) {
  BwdArgs a{};
  a.p = p;
  a.x = ar->x;
  a.rstd = (const float*)ar->rstd;
  a.x_dt = ar->x_dtype;
  a.amat = amat;
  a.nw = nwc;
  a.contig = contig;
  a.vec_ok = ((uintptr_t)ar->x % 16 == 0) && (p.C % 8 == 0);
  a.packed = packed;
  const int64_t items = (int64_t)p.Qc * ((p.BQ() + 7) / 8);
  if (items == 0) return OW_OK;
  constexpr int pack_smem = 2 * BM * 128 + STG_BYTES + (BM + D) * 4 + 128;
  auto go = [&](auto* tx) -> int {
    using TX = std::remove_pointer_t<decltype(tx)>;
    auto pk = tc_pack_kernel<D, BF16, TX, TX, true>;
    cudaError_t e = cudaFuncSetAttribute(pk, cudaFuncAttributeMaxDynamicSharedMemorySize, pack_smem);
    if (e != cudaSuccess) {
      set_error("tc forward: cannot reserve %d bytes of shared memory for the pack kernel: %s", pack_smem,
                cudaGetErrorString(e));
      return OW_ERR_CUDA;
    }
    launch(pk, (int)items, NCOMP, pack_smem, st, a);
    OW_CHECK_LAUNCH("tc_pack_kernel (forward)");
    return OW_OK;
  };
  using T16 = std::conditional_t<BF16, __nv_bfloat16, __half>;
  const int c16 = BF16 ? OW_DTYPE_BF16 : OW_DTYPE_F16;
  if (ar->x_dtype == c16) return go((T16*)nullptr);
  if (ar->x_dtype == OW_DTYPE_F32) return go((float*)nullptr);
  set_error("tc forward: unsupported x dtype %s", dtype_name(ar->x_dtype));
  return OW_ERR_UNSUPPORTED;
}
}  // namespace

int tc_pack_forward(const ow_bigemm_args_t* a, const Prob& p, const uint16_t* amat, const float* nwc,
                    const int* contig, unsigned char* packed, void* stream) {
  cudaStream_t st = (cudaStream_t)stream;
  const bool bf = a->compute_dtype == OW_DTYPE_BF16;
  if (p.d == 64)
    return bf ? tc_pack_forward_t<64, true>(a, p, amat, nwc, contig, packed, st)
              : tc_pack_forward_t<64, false>(a, p, amat, nwc, contig, packed, st);
  return bf ? tc_pack_forward_t<128, true>(a, p, amat, nwc, contig, packed, st)
            : tc_pack_forward_t<128, false>(a, p, amat, nwc, contig, packed, st);
}

int tc_backward(const ow_bigemm_args_t* a, const ow_bigemm_grads_t* gr, const Prob& p, void* stream,
                Carver& ws) {
  cudaStream_t st = (cudaStream_t)stream;
  const bool bf = a->compute_dtype == OW_DTYPE_BF16;
  if (p.d == 64) return bf ? tc_backward_t<64, true>(a, gr, p, st, ws) : tc_backward_t<64, false>(a, gr, p, st, ws);
  return bf ? tc_backward_t<128, true>(a, gr, p, st, ws) : tc_backward_t<128, false>(a, gr, p, st, ws);
}

}  // namespace ow
