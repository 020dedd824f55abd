// Tensor-core BiGEMM forward for sm_100a (bf16 / f16 compute, g = 16,
// d in {64, 128}, rd = 2d).
//
// Work unit: one channel group q_c and an "M-block" of 128 token rows (eight
// consecutive spatial tiles).  Per M-block (reference.py:147-171):
//
//   gather T (route tables, optional RMSNorm)    compute warps, registers -> smem
//   P_u = A_u T, P_v = A_v T                      compute warps, mma.sync m16n8k16
//   for each 64-wide chunk q of rd:
//     U_q = P_u B_u[:, q], V_q = P_v B_v[:, q]    tcgen05.mma, f32 in TMEM (double buffered)
//     Z_q = silu(U_q) * V_q                       compute warps, TMEM -> smem
//     Y  += Z_q B_o[q, :]                         tcgen05.mma, f32 in TMEM
//   delta = A_o Y * gamma * mask (+ x)            compute warps, mma.sync, scattered stores
//
// Roles (320 threads): warps 0-7 compute, warp 8 issues every tcgen05.mma
// (one thread) and owns the TMEM allocation, warp 9 streams pre-swizzled
// weight chunks with cp.async.bulk into a two-stage ring.  Synchronisation is
// mbarrier-only; every wait is bounded (ow_sm100.cuh).  The grid is
// persistent (one CTA per SM) and walks items channel-group-major so that the
// weight chunks of a group are shared through L2 by neighbouring CTAs.

#include <algorithm>
#include <type_traits>

#include "ow_common.cuh"
#include "ow_internal.h"
#include "ow_sm100.cuh"

namespace ow {

namespace {

using namespace sm100;

constexpr int BM = 128;                 // token rows per M-block (8 tiles of 16)
constexpr int NC = 64;                  // rd chunk width
constexpr int NCOMP_WARPS = 8;          // compute warps
constexpr int NCOMP = NCOMP_WARPS * 32;
constexpr int MMA_WARP = NCOMP_WARPS;
constexpr int PROD_WARP = NCOMP_WARPS + 1;
constexpr int TC_THREADS = (NCOMP_WARPS + 2) * 32;
constexpr int STG_LD = 72;              // staging row stride (elements): 64 + 8 pad
constexpr int TMEM_COLS = 512;

template <int D>
struct Cfg {
  static constexpr int RD = 2 * D;
  static constexpr int NQ = RD / NC;
  static constexpr int P_BYTES = BM * D * 2;
  static constexpr int Z_BYTES = BM * NC * 2;
  static constexpr int BU_BYTES = NC * D * 2;     // one of Bu/Bv chunk images
  static constexpr int WUV_BYTES = 2 * BU_BYTES;
  static constexpr int WO_BYTES = D * NC * 2;
  static constexpr int IMG_BYTES = WUV_BYTES + WO_BYTES;
  static constexpr int STG_BYTES = BM * STG_LD * 2;
  static constexpr int OFF_PU = 0;
  static constexpr int OFF_PV = OFF_PU + P_BYTES;
  static constexpr int OFF_Z = OFF_PV + P_BYTES;
  static constexpr int OFF_WUV = OFF_Z + 2 * Z_BYTES;
  static constexpr int OFF_WO = OFF_WUV + 2 * WUV_BYTES;
  static constexpr int OFF_STG = OFF_WO + 2 * WO_BYTES;
  static constexpr int OFF_META = OFF_STG + STG_BYTES;     // 2 x {tok[128], rowb[128], ch[D], gg[D], nw[D], cont}
  static constexpr int META1 = 2 * BM + 3 * D + 4;         // 32-bit words per buffer
  static constexpr int META_BYTES = 2 * META1 * 4;
  static constexpr int OFF_BAR = OFF_META + META_BYTES;
  static constexpr int BAR_BYTES = 16 * 8 + 16;
  static constexpr int SMEM = OFF_BAR + BAR_BYTES + 1024;  // + alignment slack
  // TMEM columns.
  __host__ __device__ static constexpr int T_U(int s) { return s * 128; }
  __host__ __device__ static constexpr int T_V(int s) { return s * 128 + 64; }
  static constexpr int T_Y = 256;
  static_assert(T_Y + D <= TMEM_COLS, "TMEM budget");
  static_assert(SMEM <= 232448, "shared memory budget");
};

// Workspace layout of the tensor-core path (offsets in bytes from its base).
template <int D>
struct TcWs {
  size_t img, amat, gg, nw, contig, total;
  TcWs(const Prob& p) {
    size_t o = 0;
    auto take = [&](size_t n) { size_t r = o; o = (o + n + 255) / 256 * 256; return r; };
    img = take((size_t)p.Qc * Cfg<D>::NQ * Cfg<D>::IMG_BYTES);
    amat = take(3 * 256 * 2);
    gg = take((size_t)p.Qc * D * 4);
    nw = take((size_t)p.Qc * D * 4);
    contig = take((size_t)p.Qc * 4);
    total = o;
  }
};

// ---------------------------------------------------------------------------
// Weight preparation: SW128 K-major chunk images of B_u, B_v (B operand
// [NC x D] per chunk) and B_o (B operand [D x NC] per chunk), 16-bit copies of
// the token-mix matrices, f32 grouped gamma and norm weight, and a per-group
// flag telling whether the group's channels are one aligned contiguous run.
// ---------------------------------------------------------------------------
template <int D, typename TW, bool BF16>
__global__ void tc_prep_kernel(Prob p, const TW* __restrict__ au, const TW* __restrict__ av,
                               const TW* __restrict__ ao, const TW* __restrict__ bu,
                               const TW* __restrict__ bv, const TW* __restrict__ bo,
                               const TW* __restrict__ gamma, const TW* __restrict__ nw_in,
                               unsigned char* __restrict__ img, uint16_t* __restrict__ amat,
                               float* __restrict__ gg, float* __restrict__ nw, int* __restrict__ contig) {
  using C = Cfg<D>;
  using T16 = std::conditional_t<BF16, __nv_bfloat16, __half>;
  // 32-bit indices: the divisors are compile-time constants (multiply-shift).
  constexpr int per_chunk = 3 * NC * D;
  const int n_img = p.Qc * C::NQ * per_chunk;
  const int stride = gridDim.x * blockDim.x;
  const int tid = blockIdx.x * blockDim.x + threadIdx.x;
  for (int i = tid; i < n_img; i += stride) {
    const int chunk = i / per_chunk;
    int e = i - chunk * per_chunk;
    int qc = chunk / C::NQ, q = chunk - qc * C::NQ;
    unsigned char* base = img + (int64_t)chunk * C::IMG_BYTES;
    float v;
    uint32_t off;
    if (e < 2 * NC * D) {  // Bu / Bv: row n (output feature), column k (input channel)
      int which = e / (NC * D);
      int r = e - which * NC * D;
      int n = r / D, k = r - n * D;
      const TW* src = which ? bv : bu;
      v = load_as<float>(src, ((int64_t)qc * D + k) * C::RD + q * NC + n);
      off = which * C::BU_BYTES + sw128_off(n, k, NC);
    } else {  // Bo: row n (output channel), column k (feature within chunk)
      int r = e - 2 * NC * D;
      int n = r / NC, k = r - n * NC;
      v = load_as<float>(bo, ((int64_t)qc * C::RD + q * NC + k) * D + n);
      off = C::WUV_BYTES + sw128_off(n, k, D);
    }
    *reinterpret_cast<T16*>(base + off) = Elem<T16>::from(v);
  }
  for (int i = tid; i < 3 * 256; i += stride) {
    const TW* src = i < 256 ? au : (i < 512 ? av : ao);
    T16 h = Elem<T16>::from(load_as<float>(src, i & 255));
    amat[i] = *reinterpret_cast<uint16_t*>(&h);
  }
  for (int i = tid; i < p.Qc * D; i += stride) {
    int c = p.ch[i];
    gg[i] = c < p.C ? load_as<float>(gamma, c) : 0.f;
  }
  if (nw_in)
    for (int i = tid; i < p.Qc * D; i += stride) {
      int c = p.ch[i];
      nw[i] = c < p.C ? load_as<float>(nw_in, c) : 0.f;
    }
  contig_flags<D>(p, contig);
}

// Named barrier over the compute warps only.
__device__ __forceinline__ void comp_sync() { asm volatile("bar.sync 1, %0;" ::"n"(NCOMP) : "memory"); }

template <typename TX>
__device__ __forceinline__ void load8(const TX* __restrict__ src, float (&v)[8]) {
  if constexpr (sizeof(TX) == 2) {
    uint4 u = __ldg(reinterpret_cast<const uint4*>(src));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = unpack2<std::is_same_v<TX, __nv_bfloat16>>(w[i]);
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

// ---------------------------------------------------------------------------
// Forward kernel.
// ---------------------------------------------------------------------------
template <int D, bool BF16, typename TX, typename TO>
__global__ void __launch_bounds__(TC_THREADS, 1)
tc_fwd_kernel(Prob p, const TX* __restrict__ x, const float* __restrict__ rstd, int x_dt,
              const unsigned char* __restrict__ img, const uint16_t* __restrict__ amat,
              const float* __restrict__ gg, const float* __restrict__ nw, const int* __restrict__ contig,
              const float* __restrict__ scale, int residual, TO* __restrict__ out, int vec_ok) {
  using C = Cfg<D>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  unsigned char* sPu = sm + C::OFF_PU;
  unsigned char* sPv = sm + C::OFF_PV;
  unsigned char* sZ = sm + C::OFF_Z;
  unsigned char* sWuv = sm + C::OFF_WUV;
  unsigned char* sWo = sm + C::OFF_WO;
  unsigned char* sStg = sm + C::OFF_STG;
  int* sTok = reinterpret_cast<int*>(sm + C::OFF_META);
  int* sRowB = sTok + BM;
  int* sCh = sRowB + BM;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + C::OFF_BAR);
  uint64_t* bar_p = bars + 0;
  uint64_t* bar_uv = bars + 1;   // [2]
  uint64_t* bar_z = bars + 3;    // [2]
  uint64_t* bar_yz = bars + 5;   // [2]
  uint64_t* bar_wuv = bars + 7;  // [2]
  uint64_t* bar_wo = bars + 9;   // [2]
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* sAbort = reinterpret_cast<volatile int*>(sTmem + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t BQ = (int64_t)p.B * p.Qs;
  const int nMB = (int)((BQ + 7) / 8);
  const int64_t items = (int64_t)p.Qc * nMB;
  const int my_items = items > blockIdx.x ? (int)((items - 1 - blockIdx.x) / gridDim.x + 1) : 0;

  if (threadIdx.x == 0) {
    mbar_init(bar_p, NCOMP);
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar_uv + s, 1);
      mbar_init(bar_z + s, NCOMP);
      mbar_init(bar_yz + s, 1);
      mbar_init(bar_wuv + s, 1);
      mbar_init(bar_wo + s, 1);
    }
    *sAbort = 0;
    fence_mbar_init();
  }
  if (warp == MMA_WARP) tmem_alloc(sTmem, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *sTmem;

  if (warp == PROD_WARP) {
    // ------------------------------------------------ weight producer
    if (lane == 0 && my_items > 0) {
      const int total = my_items * C::NQ;
      auto chunk_src = [&](int c) {
        int it = c / C::NQ, q = c - it * C::NQ;
        int64_t item = blockIdx.x + (int64_t)it * gridDim.x;
        int qc = (int)(item / nMB);
        return img + ((int64_t)qc * C::NQ + q) * C::IMG_BYTES;
      };
      auto load_uv = [&](int c) {
        int s = c & 1;
        mbar_arrive_expect_tx(bar_wuv + s, C::WUV_BYTES);
        bulk_g2s(sWuv + s * C::WUV_BYTES, chunk_src(c), C::WUV_BYTES, bar_wuv + s);
      };
      auto load_o = [&](int c) {
        int s = c & 1;
        mbar_arrive_expect_tx(bar_wo + s, C::WO_BYTES);
        bulk_g2s(sWo + s * C::WO_BYTES, chunk_src(c) + C::WUV_BYTES, C::WO_BYTES, bar_wo + s);
      };
      for (int c = 0; c < 2 && c < total; ++c) { load_uv(c); load_o(c); }
      for (int c = 0; c + 2 < total; ++c) {
        const int s = c & 1;
        const uint32_t ph = (c >> 1) & 1;
        if (mbar_wait(bar_uv + s, ph, sAbort)) load_uv(c + 2);
        if (mbar_wait(bar_yz + s, ph, sAbort)) load_o(c + 2);
        if (*sAbort) break;
      }
    }
  } else if (warp == MMA_WARP) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t ID_UV = idesc_f16(BM, NC, BF16);
      constexpr uint32_t ID_Y = idesc_f16(BM, D, BF16);
      const uint32_t aPu = smem_u32(sPu), aPv = smem_u32(sPv);
      int c = 0;
      auto issue_y = [&](int cy, int qy) {
        const int s = cy & 1;
        const uint32_t ph = (cy >> 1) & 1;
        mbar_wait(bar_z + s, ph, sAbort);
        mbar_wait(bar_wo + s, ph, sAbort);
        tc_fence_after();
        if (!*sAbort) {
          const uint32_t aZ = smem_u32(sZ + s * C::Z_BYTES), aW = smem_u32(sWo + s * C::WO_BYTES);
#pragma unroll
          for (int kk = 0; kk < NC / 16; ++kk)
            umma_f16(tbase + C::T_Y, sdesc_sw128(sw128_kstep(aZ, kk, BM)),
                     sdesc_sw128(sw128_kstep(aW, kk, D)), ID_Y, (qy > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(bar_yz + s);
      };
      for (int it = 0; it < my_items; ++it) {
        mbar_wait(bar_p, it & 1, sAbort);
        tc_fence_after();
        for (int q = 0; q < C::NQ; ++q, ++c) {
          const int s = c & 1;
          const uint32_t ph = (c >> 1) & 1;
          mbar_wait(bar_wuv + s, ph, sAbort);
          tc_fence_after();
          if (!*sAbort) {
            const uint32_t aBu = smem_u32(sWuv + s * C::WUV_BYTES);
            const uint32_t aBv = aBu + C::BU_BYTES;
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              umma_f16(tbase + C::T_U(s), sdesc_sw128(sw128_kstep(aPu, kk, BM)),
                       sdesc_sw128(sw128_kstep(aBu, kk, NC)), ID_UV, kk > 0 ? 1u : 0u);
              umma_f16(tbase + C::T_V(s), sdesc_sw128(sw128_kstep(aPv, kk, BM)),
                       sdesc_sw128(sw128_kstep(aBv, kk, NC)), ID_UV, kk > 0 ? 1u : 0u);
            }
          }
          umma_commit(bar_uv + s);
          if (q >= 1) issue_y(c - 1, q - 1);
        }
        issue_y(c - 1, C::NQ - 1);
      }
    }
  } else {
    // ------------------------------------------------ compute warps
    const int tid = threadIdx.x;
    const int g = lane >> 2, t4 = lane & 3;
    // Token-mix matrices as m16n8k16 A fragments.
    uint32_t fa[3][4];
#pragma unroll
    for (int m = 0; m < 3; ++m) {
      const uint16_t* A = amat + m * 256;
      fa[m][0] = *reinterpret_cast<const uint32_t*>(A + g * 16 + 2 * t4);
      fa[m][1] = *reinterpret_cast<const uint32_t*>(A + (g + 8) * 16 + 2 * t4);
      fa[m][2] = *reinterpret_cast<const uint32_t*>(A + g * 16 + 2 * t4 + 8);
      fa[m][3] = *reinterpret_cast<const uint32_t*>(A + (g + 8) * 16 + 2 * t4 + 8);
    }
    const uint32_t aStg = smem_u32(sStg);
    int32_t* meta = reinterpret_cast<int32_t*>(sTok);
    auto mTok = [&](int buf) { return meta + buf * C::META1; };
    auto mRowB = [&](int buf) { return meta + buf * C::META1 + BM; };
    auto mCh = [&](int buf) { return meta + buf * C::META1 + 2 * BM; };
    auto mGG = [&](int buf) { return reinterpret_cast<float*>(meta + buf * C::META1 + 2 * BM + D); };
    auto mNW = [&](int buf) { return reinterpret_cast<float*>(meta + buf * C::META1 + 2 * BM + 2 * D); };
    auto mCont = [&](int buf) { return meta + buf * C::META1 + 2 * BM + 3 * D; };

    // Metadata of one item, held in registers between issue and store.  The
    // loads are unconditional (clamped indices) and their values are first
    // used in meta_store, so issuing them does not wait for memory.
    struct MetaReg { int tok, b, ch, cont; float gg, nw; bool valid; };
    auto meta_issue = [&](int it) {
      MetaReg m{0, 0, 0, 0, 0.f, 0.f, false};
      const int64_t item = blockIdx.x + (int64_t)it * gridDim.x;
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
      if (tid < D) {
        m.ch = p.ch[qc * D + tid];
        m.gg = gg[(int64_t)qc * D + tid];
        if (rstd) m.nw = nw[(int64_t)qc * D + tid];
      }
      if (tid == 0) m.cont = contig[qc];
      return m;
    };
    auto meta_store = [&](const MetaReg& m, int buf) {
      if (tid < BM) {
        mTok(buf)[tid] = m.valid && m.tok < p.N ? m.tok : -1;
        mRowB(buf)[tid] = m.b;
      }
      if (tid < D) { mCh(buf)[tid] = m.ch; mGG(buf)[tid] = m.gg; mNW(buf)[tid] = m.nw; }
      if (tid == 0) *mCont(buf) = vec_ok && m.cont != 0;
    };

    // Gathered rows of one 64-channel half, held in registers (contiguous path).
    constexpr int VW = sizeof(TX) == 2 ? 1 : 2;  // 16-byte vectors per 8 elements
    struct RowReg { uint4 v[4][VW]; float rs[4]; };
    auto rows_issue = [&](RowReg& R, int buf, int hf) {
      const int* tk = mTok(buf);
      const int* rb = mRowB(buf);
      const int ch0 = mCh(buf)[0];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int unit = tid + u * NCOMP;
        const int r = unit >> 3, cj = unit & 7;
        // Pad rows load row 0 (always valid) and are zeroed in rows_store;
        // no value is used here, so the loads stay in flight.
        const int tok = tk[r] >= 0 ? tk[r] : 0;
        const int64_t row = (int64_t)rb[r] * p.N + tok;
        const uint4* src = reinterpret_cast<const uint4*>(x + row * p.C + ch0 + hf * 64 + cj * 8);
#pragma unroll
        for (int vv = 0; vv < VW; ++vv) R.v[u][vv] = __ldg(src + vv);
        R.rs[u] = rstd ? rstd[row] : 1.f;
      }
    };
    auto rows_store = [&](const RowReg& R, int buf, int hf) {
      const float* nwq = mNW(buf);
      const int* tk = mTok(buf);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int unit = tid + u * NCOMP;
        const int r = unit >> 3, cj = unit & 7;
        const bool pad = tk[r] < 0;
        float v[8];
        if constexpr (sizeof(TX) == 2) {
          const uint32_t w[4] = {R.v[u][0].x, R.v[u][0].y, R.v[u][0].z, R.v[u][0].w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float2 f = unpack2<std::is_same_v<TX, __nv_bfloat16>>(w[i]);
            v[2 * i] = f.x;
            v[2 * i + 1] = f.y;
          }
        } else {
#pragma unroll
          for (int vv = 0; vv < 2; ++vv) {
            v[4 * vv + 0] = __uint_as_float(R.v[u][vv].x);
            v[4 * vv + 1] = __uint_as_float(R.v[u][vv].y);
            v[4 * vv + 2] = __uint_as_float(R.v[u][vv].z);
            v[4 * vv + 3] = __uint_as_float(R.v[u][vv].w);
          }
        }
        if (rstd) {
          const int k0 = hf * 64 + cj * 8;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            float t = round_through(v[e] * R.rs[u], x_dt);
            v[e] = round_through(t * nwq[k0 + e], x_dt);
          }
        }
        if (pad) {
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] = 0.f;
        }
        uint4 w;
        w.x = pack2<BF16>(v[0], v[1]);
        w.y = pack2<BF16>(v[2], v[3]);
        w.z = pack2<BF16>(v[4], v[5]);
        w.w = pack2<BF16>(v[6], v[7]);
        *reinterpret_cast<uint4*>(sStg + (r * STG_LD + cj * 8) * 2) = w;
      }
    };
    // Element-wise gather (channels not one aligned run): synchronous.
    auto rows_elem = [&](int buf, int hf) {
      const int* tk = mTok(buf);
      const int* rb = mRowB(buf);
      const int* chs = mCh(buf);
      const float* nwq = mNW(buf);
      for (int e = tid; e < BM * 64; e += NCOMP) {
        const int r = e >> 6, k = e & 63;
        const int tok = tk[r], ch = chs[hf * 64 + k];
        float v = 0.f;
        if (tok >= 0 && ch < p.C) {
          const int64_t row = (int64_t)rb[r] * p.N + tok;
          v = load_as<float>(x, row * p.C + ch);
          if (rstd) {
            v = round_through(v * rstd[row], x_dt);
            v = round_through(v * nwq[hf * 64 + k], x_dt);
          }
        }
        uint32_t pk = pack2<BF16>(v, 0.f);
        *reinterpret_cast<uint16_t*>(sStg + (r * STG_LD + k) * 2) = (uint16_t)(pk & 0xFFFF);
      }
    };

    RowReg R;
    MetaReg mnext{};
    if (my_items > 0) {
      meta_store(meta_issue(0), 0);
      comp_sync();
      if (*mCont(0)) rows_issue(R, 0, 0);
      if (my_items > 1) mnext = meta_issue(1);
    }
    int c = 0;
    for (int it = 0; it < my_items; ++it) {
      const int buf = it & 1;
      const bool cont = *mCont(buf) != 0;
      const int* sTk = mTok(buf);
      const int* sRb = mRowB(buf);
      const int* sChs = mCh(buf);
      const float* sG = mGG(buf);
      const int ch0 = sChs[0];

      if (tid == 0 && it < 3) OW_TR(0, it * 32 + 0);
      // -------- gather + token mix, 64 channels at a time
      for (int hf = 0; hf < D / 64; ++hf) {
        if (cont) {
          rows_store(R, buf, hf);
          if (hf + 1 < D / 64) rows_issue(R, buf, hf + 1);
        } else {
          rows_elem(buf, hf);
        }
        comp_sync();
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_trans(aStg + ((warp * 16 + (lane & 15)) * STG_LD + np * 16 + (lane >> 4) * 8) * 2, b0, b1, b2,
                        b3);
#pragma unroll
          for (int m = 0; m < 2; ++m) {
            float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
            mma16816<BF16>(c0, fa[m], b0, b1);
            mma16816<BF16>(c1, fa[m], b2, b3);
            unsigned char* P = m ? sPv : sPu;
            const int r0 = warp * 16 + g, k0 = hf * 64 + np * 16 + 2 * t4;
            *reinterpret_cast<uint32_t*>(P + sw128_off(r0, k0, BM)) = pack2<BF16>(c0[0], c0[1]);
            *reinterpret_cast<uint32_t*>(P + sw128_off(r0 + 8, k0, BM)) = pack2<BF16>(c0[2], c0[3]);
            *reinterpret_cast<uint32_t*>(P + sw128_off(r0, k0 + 8, BM)) = pack2<BF16>(c1[0], c1[1]);
            *reinterpret_cast<uint32_t*>(P + sw128_off(r0 + 8, k0 + 8, BM)) = pack2<BF16>(c1[2], c1[3]);
          }
        }
        comp_sync();  // staging reused by the next half
      }
      fence_proxy_async_smem();
      if (tid == 0 && it < 3) OW_TR(0, it * 32 + 1);
      mbar_arrive(bar_p);

      // -------- gate: Z_q = silu(U_q) * V_q
      const int lq = warp & 3, cb = (warp >> 2) * 32;
      const int r = lq * 32 + lane;
      const uint32_t trow = tbase + ((uint32_t)(lq * 32) << 16);
      for (int q = 0; q < C::NQ; ++q, ++c) {
        const int s = c & 1;
        const uint32_t ph = (c >> 1) & 1;
        mbar_wait(bar_uv + s, ph, sAbort);
        if (tid == 0 && it < 3 && q < 4) OW_TR(0, it * 32 + 2 + 2 * q);
        __syncwarp();
        tc_fence_after();
        uint32_t ur[32], vr[32];
        tmem_ld32(trow + C::T_U(s) + cb, ur);
        tmem_ld32(trow + C::T_V(s) + cb, vr);
        tmem_ld_wait();
        if (c >= 2) mbar_wait(bar_yz + s, ((c - 2) >> 1) & 1, sAbort);
        unsigned char* Zs = sZ + s * C::Z_BYTES;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          uint4 w;
          uint32_t* wp = &w.x;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int i0 = jj * 8 + 2 * e;
            uint32_t u2 = pack2<BF16>(__uint_as_float(ur[i0]), __uint_as_float(ur[i0 + 1]));
            uint32_t v2 = pack2<BF16>(__uint_as_float(vr[i0]), __uint_as_float(vr[i0 + 1]));
            wp[e] = silu_mul2<BF16>(u2, v2);
          }
          *reinterpret_cast<uint4*>(Zs + sw128_off(r, cb + jj * 8, BM)) = w;
        }
        fence_proxy_async_smem();
        tc_fence_before();
        if (tid == 0 && it < 3 && q < 4) OW_TR(0, it * 32 + 3 + 2 * q);
        mbar_arrive(bar_z + s);
      }

      // -------- prefetch the next item's metadata and first half of rows
      if (it + 1 < my_items) {
        meta_store(mnext, buf ^ 1);
        if (tid == 0 && it < 3) OW_TR(0, it * 32 + 20);
        comp_sync();
        if (tid == 0 && it < 3) OW_TR(0, it * 32 + 21);
        if (*mCont(buf ^ 1)) rows_issue(R, buf ^ 1, 0);
        if (tid == 0 && it < 3) OW_TR(0, it * 32 + 22);
        if (it + 2 < my_items) mnext = meta_issue(it + 2);
        if (tid == 0 && it < 3) OW_TR(0, it * 32 + 23);
      }

      // -------- epilogue: delta = A_o Y, gamma, mask, residual, scatter
      if (tid == 0 && it < 3) OW_TR(0, it * 32 + 12);
      mbar_wait(bar_yz + ((c - 1) & 1), ((c - 1) >> 1) & 1, sAbort);
      if (tid == 0 && it < 3) OW_TR(0, it * 32 + 13);
      __syncwarp();
      tc_fence_after();
      for (int hf = 0; hf < D / 64; ++hf) {
        uint32_t yr[32];
        tmem_ld32(trow + C::T_Y + hf * 64 + cb, yr);
        tmem_ld_wait();
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          uint4 w;
          w.x = pack2<BF16>(__uint_as_float(yr[jj * 8 + 0]), __uint_as_float(yr[jj * 8 + 1]));
          w.y = pack2<BF16>(__uint_as_float(yr[jj * 8 + 2]), __uint_as_float(yr[jj * 8 + 3]));
          w.z = pack2<BF16>(__uint_as_float(yr[jj * 8 + 4]), __uint_as_float(yr[jj * 8 + 5]));
          w.w = pack2<BF16>(__uint_as_float(yr[jj * 8 + 6]), __uint_as_float(yr[jj * 8 + 7]));
          *reinterpret_cast<uint4*>(sPu + (r * STG_LD + cb + jj * 8) * 2) = w;
        }
        comp_sync();
        const int row0 = warp * 16 + g;
        const int tokA = sTk[row0], tokB = sTk[row0 + 8];
        const int bA = sRb[row0], bB = sRb[row0 + 8];
        const float sA = scale ? scale[bA] : 1.f, sB = scale ? scale[bB] : 1.f;
        const uint32_t aEp = smem_u32(sPu);
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          __syncwarp();
          uint32_t b0, b1, b2, b3;
          ldsm_x4_trans(aEp + ((warp * 16 + (lane & 15)) * STG_LD + np * 16 + (lane >> 4) * 8) * 2, b0, b1, b2,
                        b3);
          float cc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
          mma16816<BF16>(cc[0], fa[2], b0, b1);
          mma16816<BF16>(cc[1], fa[2], b2, b3);
#pragma unroll
          for (int nb = 0; nb < 2; ++nb) {
            const int k = hf * 64 + np * 16 + nb * 8 + 2 * t4;
            const float g0 = sG[k], g1 = sG[k + 1];
#pragma unroll
            for (int hr = 0; hr < 2; ++hr) {
              const int tok = hr ? tokB : tokA;
              if (tok < 0) continue;
              const int64_t row = (int64_t)(hr ? bB : bA) * p.N + tok;
              const float sc = hr ? sB : sA;
              float d0 = cc[nb][2 * hr] * g0 * sc;
              float d1 = cc[nb][2 * hr + 1] * g1 * sc;
              if (cont) {
                const int64_t off = row * p.C + ch0 + k;
                if (residual) {
                  d0 += load_as<float>(x, off);
                  d1 += load_as<float>(x, off + 1);
                }
                if constexpr (std::is_same_v<TO, float>) {
                  *reinterpret_cast<float2*>(out + off) = make_float2(d0, d1);
                } else {
                  *reinterpret_cast<uint32_t*>(out + off) =
                      pack2<std::is_same_v<TO, __nv_bfloat16>>(d0, d1);
                }
              } else {
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                  const int ch = sChs[k + e];
                  if (ch >= p.C) continue;
                  const int64_t off = row * p.C + ch;
                  float dv = e ? d1 : d0;
                  if (residual) dv += load_as<float>(x, off);
                  out[off] = Elem<TO>::from(dv);
                }
              }
            }
          }
        }
        comp_sync();
      }
      if (tid == 0 && it < 3) OW_TR(0, it * 32 + 14);
      tc_fence_before();
    }
  }

  __syncwarp();
  __syncthreads();
  if (*sAbort) {
    // A wait gave up: give in-flight copies and MMAs time to land before
    // the shared memory and TMEM they target are released.
    for (int i = 0; i < 1000; ++i) __nanosleep(1000);
  }
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tbase, TMEM_COLS);
  }
}

int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!cached[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

template <int D, bool BF16>
int tc_prep(const ow_bigemm_args_t* a, const Prob& p, const TcWs<D>& w, unsigned char* base,
            cudaStream_t st) {
  const int64_t n = 3LL * p.Qc * D * 2 * D;
  const int grid = (int)std::min<int64_t>((n + 255) / 256, 148 * 8);
  auto run = [&](auto* tw) {
    using TW = std::remove_pointer_t<decltype(tw)>;
    launch(tc_prep_kernel<D, TW, BF16>, grid, 256, 0, st, p, (const TW*)a->a_u, (const TW*)a->a_v,
           (const TW*)a->a_o, (const TW*)a->b_u, (const TW*)a->b_v, (const TW*)a->b_o,
           (const TW*)a->gamma, (const TW*)(a->rstd ? a->norm_w : nullptr), base + w.img,
           (uint16_t*)(base + w.amat), (float*)(base + w.gg), (float*)(base + w.nw),
           (int*)(base + w.contig));
  };
  switch (a->w_dtype) {
    case OW_DTYPE_F32: run((float*)nullptr); break;
    case OW_DTYPE_F64: run((double*)nullptr); break;
    case OW_DTYPE_BF16: run((__nv_bfloat16*)nullptr); break;
    case OW_DTYPE_F16: run((__half*)nullptr); break;
    default: set_error("unsupported weight dtype"); return OW_ERR_UNSUPPORTED;
  }
  OW_CHECK_LAUNCH("tc_prep_kernel");
  return OW_OK;
}

template <int D, bool BF16>
int tc_forward_t(const ow_bigemm_args_t* a, const Prob& p, cudaStream_t st, Carver& ws) {
  TcWs<D> w(p);
  unsigned char* base = (unsigned char*)ws.take(w.total);
  if (!ws.base) return OW_OK;
  OW_RETURN_IF((tc_prep<D, BF16>(a, p, w, base, st)));
  const int64_t items = (int64_t)p.Qc * ((p.BQ() + 7) / 8);
  const int grid = (int)std::min<int64_t>(items, num_sms());
  // 16-byte vector loads/stores need aligned bases (channel runs are checked
  // per group by the prep kernel).
  const int vec_ok = ((uintptr_t)a->x % 16 == 0) && ((uintptr_t)a->out % 16 == 0) && (p.C % 8 == 0);
  auto go = [&](auto* tx, auto* to) -> int {
    using TX = std::remove_pointer_t<decltype(tx)>;
    using TO = std::remove_pointer_t<decltype(to)>;
    auto kern = tc_fwd_kernel<D, BF16, TX, TO>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<D>::SMEM);
    if (e != cudaSuccess) {
      set_error("tc forward: cannot reserve %d bytes of shared memory: %s", Cfg<D>::SMEM, cudaGetErrorString(e));
      return OW_ERR_CUDA;
    }
    profile_mark(OW_PROF_FWD, false, st);
    launch(kern, grid, TC_THREADS, Cfg<D>::SMEM, st, p, (const TX*)a->x, (const float*)a->rstd, a->x_dtype,
           (const unsigned char*)(base + w.img), (const uint16_t*)(base + w.amat),
           (const float*)(base + w.gg), (const float*)(base + w.nw), (const int*)(base + w.contig),
           a->sample_scale, a->residual, (TO*)a->out, vec_ok);
    profile_mark(OW_PROF_FWD, true, st);
    OW_CHECK_LAUNCH("tc_fwd_kernel");
    return OW_OK;
  };
  using T16 = std::conditional_t<BF16, __nv_bfloat16, __half>;
  const int xd = a->x_dtype, od = a->out_dtype;
  const int c16 = BF16 ? OW_DTYPE_BF16 : OW_DTYPE_F16;
  if (xd == c16 && od == c16) return go((T16*)nullptr, (T16*)nullptr);
  if (xd == c16 && od == OW_DTYPE_F32) return go((T16*)nullptr, (float*)nullptr);
  if (xd == OW_DTYPE_F32 && od == OW_DTYPE_F32) return go((float*)nullptr, (float*)nullptr);
  if (xd == OW_DTYPE_F32 && od == c16) return go((float*)nullptr, (T16*)nullptr);
  set_error("tc forward: unsupported dtypes x=%s out=%s", dtype_name(xd), dtype_name(od));
  return OW_ERR_UNSUPPORTED;
}

}  // namespace

int tc_fault(int device, int reset) {
  int prev = 0, v = 0;
  cudaGetDevice(&prev);
  if (cudaSetDevice(device) != cudaSuccess) return -1;
  if (cudaMemcpyFromSymbol(&v, sm100::g_fault, sizeof(int)) != cudaSuccess) v = -1;
  if (reset && v > 0) {
    int z = 0;
    cudaMemcpyToSymbol(sm100::g_fault, &z, sizeof(int));
  }
  cudaSetDevice(prev);
  return v;
}

bool tc_supported(const ow_bigemm_args_t* a, const Prob& p, const char** why) {
  auto no = [&](const char* m) {
    if (why) *why = m;
    return false;
  };
  if (a->compute_dtype != OW_DTYPE_BF16 && a->compute_dtype != OW_DTYPE_F16) return no("compute dtype");
  if (p.g != 16) return no("g != 16");
  if (!((p.d == 64 || p.d == 128) && p.rd == 2 * p.d)) return no("tile shape");
  const int c16 = a->compute_dtype;
  if (a->x_dtype != c16 && a->x_dtype != OW_DTYPE_F32) return no("x dtype");
  if (a->out_dtype != c16 && a->out_dtype != OW_DTYPE_F32 && a->out != nullptr) return no("out dtype");
  if (a->rstd && a->compute_dtype == OW_DTYPE_F64) return no("rstd dtype");
  return true;
}

int tc_forward(const ow_bigemm_args_t* a, const Prob& p, void* stream, Carver& ws) {
  cudaStream_t st = (cudaStream_t)stream;
  const bool bf = a->compute_dtype == OW_DTYPE_BF16;
  if (p.d == 64) return bf ? tc_forward_t<64, true>(a, p, st, ws) : tc_forward_t<64, false>(a, p, st, ws);
  return bf ? tc_forward_t<128, true>(a, p, st, ws) : tc_forward_t<128, false>(a, p, st, ws);
}

}  // namespace ow

#ifdef OW_TRACE
extern "C" __attribute__((visibility("default"))) int ow_trace_fwd(void* host, size_t bytes, int clear) {
  if (clear) {
    void* dev = nullptr;
    cudaGetSymbolAddress(&dev, ow::sm100::g_trace);
    return (int)cudaMemset(dev, 0, sizeof(ow::sm100::g_trace));
  }
  return (int)cudaMemcpyFromSymbol(host, ow::sm100::g_trace, bytes);
}
#endif
