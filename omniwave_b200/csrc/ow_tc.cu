// Tensor-core BiGEMM forward for sm_100a (bf16 / f16 compute, g = 16,
// d in {64, 128}, rd = 2d).
//
// Work unit ("item"): one channel group q_c and an M-block of 128 token rows
// (eight consecutive spatial tiles).  Per item (reference.py:147-171):
//
//   gather T (route tables, optional RMSNorm)    pack kernel (ow_tc_bwd.cu), one CTA per item
//   P_u = A_u T, P_v = A_v T                      pack kernel, mma.sync, SW128 images in HBM
//   for each 64-wide chunk q of rd:               forward kernel (this file):
//     U_q = P_u B_u[:, q], V_q = P_v B_v[:, q]    tcgen05.mma, f32 in TMEM (double buffered)
//     Z_q = silu(U_q) * V_q                       compute warps, TMEM -> smem
//     Y  += Z_q B_o[q, :]                         tcgen05.mma, f32 in TMEM
//   delta = A_o Y * gamma * scale (+ x)           compute warps: TMEM C-fragments, mma.sync,
//                                                 f32 staging, full-line row stores
//
// Roles of the forward kernel (320 threads): warps 0-7 compute, warp 8 issues
// every tcgen05.mma (one thread) and owns the TMEM allocation, warp 9 issues
// the bulk copies: the packed [P_u | P_v] of each item (two item buffers at
// d = 64, one at d = 128) and the pre-swizzled weight chunk images (resident
// per channel group at d = 64, a two-stage ring at d = 128).  The epilogue's
// warp MMAs run while the tensor pipe is idle (the next item's second chunk
// waits for it): mma.sync latency rises tenfold behind queued tcgen05 work.
// Synchronisation is mbarrier-only; every wait is bounded (ow_sm100.cuh).
// The grid is persistent (one CTA per SM) and walks items
// channel-group-major so that the weight chunks of a group are shared
// through L2 by neighbouring CTAs.

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
constexpr int TMEM_COLS = 512;

template <int D>
struct Cfg {
  static constexpr int RD = 2 * D;
  static constexpr int NQ = RD / NC;
  static constexpr int P_BYTES = BM * D * 2;
  static constexpr int PP_BYTES = 2 * P_BYTES;           // [P_u | P_v] of one item
  static constexpr int ROWS_BYTES = BM * 4;              // output row of each token row (-1: none)
  static constexpr int PK_BYTES = PP_BYTES + ROWS_BYTES;  // one item of the packed buffer
  static constexpr int Z_BYTES = BM * NC * 2;
  static constexpr int BU_BYTES = NC * D * 2;            // one of Bu/Bv chunk images
  static constexpr int WUV_BYTES = 2 * BU_BYTES;
  static constexpr int WO_BYTES = D * NC * 2;
  static constexpr int IMG_BYTES = WUV_BYTES + WO_BYTES;
  static constexpr int GRP_BYTES = NQ * IMG_BYTES;       // chunk images of one channel group
  // d = 64: two groups of chunk images (48 KB each) stay resident (the next
  // group's arrives while the current one is in use), the item operands are
  // double-buffered, and the compute warps run the next item's first gate
  // before this item's epilogue.  d = 128: the chunk images stream through a
  // two-stage ring, one item buffer, gates then epilogue.
  static constexpr bool RES = D == 64;
  static constexpr int NB = RES ? 2 : 1;
  static constexpr int OFF_P = 0;
  static constexpr int OFF_Z = OFF_P + NB * PP_BYTES;
  static constexpr int OFF_W = OFF_Z + 2 * Z_BYTES;       // resident: 2 x GRP_BYTES
  static constexpr int OFF_WUV = OFF_W;                   // streaming: 2 x [Bu | Bv]
  static constexpr int OFF_WO = OFF_WUV + 2 * WUV_BYTES;  // streaming: 2 x Bo
  static constexpr int W_END = RES ? OFF_W + 2 * GRP_BYTES : OFF_WO + 2 * WO_BYTES;
  static constexpr int OFF_ROWS = W_END;                  // 2 x ROWS_BYTES
  static constexpr int ST_LD = 72;                         // epilogue staging row stride (f32): 64 + 8 pad
  static constexpr int STG_WARP = 8 * ST_LD * 4;           // per compute warp: 8 rows x 64 channels
  static constexpr int OFF_STG = OFF_ROWS + 2 * ROWS_BYTES;
  static constexpr int OFF_BAR = OFF_STG + 8 * STG_WARP;
  static constexpr int NBAR = 23;
  static constexpr int BAR_BYTES = NBAR * 8 + 16;
  static constexpr int SMEM = OFF_BAR + BAR_BYTES + 1024;  // + alignment slack
  // TMEM columns: U/V of two chunks, Y of two items.
  __host__ __device__ static constexpr int T_U(int s) { return s * 128; }
  __host__ __device__ static constexpr int T_V(int s) { return s * 128 + 64; }
  __host__ __device__ static constexpr int T_Y(int b) { return 256 + b * D; }
  static_assert(256 + 2 * D <= TMEM_COLS, "TMEM budget");
  static_assert(SMEM <= 232448, "shared memory budget");
};

// Workspace layout of the tensor-core path (offsets in bytes from its base).
template <int D>
struct TcWs {
  size_t img, amat, gg, nwc, contig, packed, total;
  // ``gather``: the call runs the TMA-gather forward (ow_tcf.cu), which
  // needs no packed operand images.
  TcWs(const Prob& p, bool gather) {
    size_t o = 0;
    auto take = [&](size_t n) { size_t r = o; o = (o + n + 255) / 256 * 256; return r; };
    img = take((size_t)p.Qc * Cfg<D>::NQ * Cfg<D>::IMG_BYTES);
    amat = take(3 * 256 * 2);
    gg = take((size_t)p.Qc * D * 4);
    nwc = take((size_t)p.C * 4);
    contig = take((size_t)p.Qc * 4);
    packed = gather ? 0 : take((size_t)p.Qc * ((p.BQ() + 7) / 8) * Cfg<D>::PK_BYTES);
    total = o;
  }
};

// ---------------------------------------------------------------------------
// Weight preparation: SW128 K-major chunk images of B_u, B_v (B operand
// [NC x D] per chunk) and B_o (B operand [D x NC] per chunk), 16-bit copies of
// the token-mix matrices, f32 grouped gamma, the f32 norm weight per channel,
// and a per-group flag telling whether the group's channels are one aligned
// contiguous run.
// ---------------------------------------------------------------------------
template <int D, typename TW, bool BF16>
__global__ void tc_prep_kernel(Prob p, const TW* __restrict__ au, const TW* __restrict__ av,
                               const TW* __restrict__ ao, const TW* __restrict__ bu,
                               const TW* __restrict__ bv, const TW* __restrict__ bo,
                               const TW* __restrict__ gamma, const TW* __restrict__ nw_in,
                               unsigned char* __restrict__ img, uint16_t* __restrict__ amat,
                               float* __restrict__ gg, float* __restrict__ nwc,
                               int* __restrict__ contig) {
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
    for (int i = tid; i < p.C; i += stride) nwc[i] = load_as<float>(nw_in, i);
  contig_flags<D>(p, contig);
}

// ---------------------------------------------------------------------------
// Forward kernel.  [P_u | P_v] and the output rows of every item come
// pre-packed (pack pass) and arrive by bulk copy; the compute warps run the
// gates and the epilogue only.
// ---------------------------------------------------------------------------
template <int D, bool BF16, typename TX, typename TO>
__global__ void __launch_bounds__(TC_THREADS, 1)
tc_fwd_kernel(Prob p, const TX* __restrict__ x, const unsigned char* __restrict__ packed,
              const unsigned char* __restrict__ img, const uint16_t* __restrict__ amat,
              const float* __restrict__ gg, const int* __restrict__ contig, const float* __restrict__ scale,
              int residual, TO* __restrict__ out, int vec_ok, int* fault, uint32_t probe_ns) {
  using C = Cfg<D>;
  constexpr bool EARLY = C::RES;  // next item's first gate before this item's epilogue
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  unsigned char* sZ = sm + C::OFF_Z;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + C::OFF_BAR);
  uint64_t* bar_p = bars + 0;       // [2] item operands of item buffer i loaded (tx)
  uint64_t* bar_uv = bars + 2;      // [2] U/V of TMEM buffer s computed (commit)
  uint64_t* bar_z = bars + 4;       // [2] Z_s written, TMEM buffer s read
  uint64_t* bar_yz = bars + 6;      // [2] Y MMA of Z buffer s done (commit)
  uint64_t* bar_wuv = bars + 8;     // [2] streaming: [B_u | B_v] stage loaded (tx)
  uint64_t* bar_wo = bars + 10;     // [2] streaming: B_o stage loaded (tx)
  uint64_t* bar_pf = bars + 12;     // [2] operands of item buffer i no longer read (commit)
  uint64_t* bar_epd = bars + 14;    // [2] epilogue of an item with parity b done
  uint64_t* bar_wres = bars + 16;   // [2] resident: chunk images of group buffer b loaded (tx)
  uint64_t* bar_wfree = bars + 18;  // [2] resident: group buffer b no longer read (commit)
  uint64_t* bar_m = bars + 20;      // [2] output rows of row slot b loaded (tx)
  uint64_t* bar_probe = bars + 22;  // wait-timeout self-check: nothing arrives on it
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(bars + C::NBAR);
  volatile int* sAbort = reinterpret_cast<volatile int*>(sTmem + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t BQ = (int64_t)p.B * p.Qs;
  const int nMB = (int)((BQ + 7) / 8);
  const int64_t items = (int64_t)p.Qc * nMB;
  const int nit = items > blockIdx.x ? (int)((items - 1 - blockIdx.x) / gridDim.x + 1) : 0;
  const int total = nit * C::NQ;
  auto item_of = [&](int it) { return (int64_t)blockIdx.x + (int64_t)it * gridDim.x; };
  auto qc_of = [&](int it) { return (int)(item_of(it) / nMB); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar_p + s, 1);
      mbar_init(bar_uv + s, 1);
      mbar_init(bar_z + s, NCOMP);
      mbar_init(bar_yz + s, 1);
      mbar_init(bar_wuv + s, 1);
      mbar_init(bar_wo + s, 1);
      mbar_init(bar_pf + s, 1);
      mbar_init(bar_epd + s, NCOMP);
      mbar_init(bar_wres + s, 1);
      mbar_init(bar_wfree + s, 1);
      mbar_init(bar_m + s, 1);
    }
    mbar_init(bar_probe, 1);
    *sAbort = 0;
    fence_mbar_init();
    wait_probe(bar_probe, sAbort, probe_ns);
  }
  if (warp == MMA_WARP) tmem_alloc(sTmem, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *sTmem;

  if (*sAbort) {
    // The wait-timeout self-check ran out before any work was issued.
  } else if (warp == PROD_WARP) {
    // ------------------------------------------------ producer (bulk copies)
    if (lane == 0 && nit > 0) {
      auto load_p = [&](int it) {
        const int bf = it % C::NB;
        mbar_arrive_expect_tx(bar_p + bf, C::PP_BYTES);
        bulk_g2s(sm + C::OFF_P + bf * C::PP_BYTES, packed + item_of(it) * C::PK_BYTES, C::PP_BYTES, bar_p + bf);
      };
      // Output rows of item it into row slot it & 1, once the epilogue of
      // item it - 2 (the slot's last reader) is done.
      auto load_rows = [&](int it) {
        const int sl = it & 1;
        if (it >= 2 && !mbar_wait(bar_epd + sl, ((it - 2) >> 1) & 1, sAbort)) return;
        mbar_arrive_expect_tx(bar_m + sl, C::ROWS_BYTES);
        bulk_g2s(sm + C::OFF_ROWS + sl * C::ROWS_BYTES, packed + item_of(it) * C::PK_BYTES + C::PP_BYTES,
                 C::ROWS_BYTES, bar_m + sl);
      };
      if constexpr (C::RES) {
        // Group e (a run of items of one channel group) uses buffer e & 1; it
        // is loaded once group e - 2 has released that buffer.
        int we = 0, wq = qc_of(0);
        auto load_w = [&](int e, int qc) {
          const int b = e & 1;
          if (e >= 2 && !mbar_wait(bar_wfree + b, ((e - 2) >> 1) & 1, sAbort)) return;
          mbar_arrive_expect_tx(bar_wres + b, C::GRP_BYTES);
          bulk_g2s(sm + C::OFF_W + b * C::GRP_BYTES, img + (int64_t)qc * C::GRP_BYTES, C::GRP_BYTES, bar_wres + b);
        };
        load_w(0, wq);
        load_p(0);
        load_rows(0);
        if (nit > 1) {
          load_p(1);
          load_rows(1);
          if (qc_of(1) != wq) load_w(++we, wq = qc_of(1));
        }
        for (int it = 0; it + 2 < nit && !*sAbort; ++it) {
          if (mbar_wait(bar_pf + (it & 1), (it >> 1) & 1, sAbort)) load_p(it + 2);
          if (qc_of(it + 2) != wq) load_w(++we, wq = qc_of(it + 2));
          load_rows(it + 2);
        }
      } else {
        auto chunk_src = [&](int c) {
          const int it = c / C::NQ, q = c - it * C::NQ;
          return img + ((int64_t)qc_of(it) * C::NQ + q) * C::IMG_BYTES;
        };
        auto load_uv = [&](int c) {
          const int s = c & 1;
          mbar_arrive_expect_tx(bar_wuv + s, C::WUV_BYTES);
          bulk_g2s(sm + C::OFF_WUV + s * C::WUV_BYTES, chunk_src(c), C::WUV_BYTES, bar_wuv + s);
        };
        auto load_o = [&](int c) {
          const int s = c & 1;
          mbar_arrive_expect_tx(bar_wo + s, C::WO_BYTES);
          bulk_g2s(sm + C::OFF_WO + s * C::WO_BYTES, chunk_src(c) + C::WUV_BYTES, C::WO_BYTES, bar_wo + s);
        };
        load_p(0);
        load_rows(0);
        if (nit > 1) load_rows(1);
        for (int c = 0; c < 2 && c < total; ++c) {
          load_uv(c);
          load_o(c);
        }
        for (int c = 0; c < total && !*sAbort; ++c) {
          const int it = c / C::NQ, q = c - it * C::NQ;
          const int s = c & 1;
          const uint32_t ph = (c >> 1) & 1;
          if (c + 2 < total && mbar_wait(bar_uv + s, ph, sAbort)) load_uv(c + 2);
          if (q == C::NQ - 1 && it + 1 < nit && mbar_wait(bar_pf, it & 1, sAbort)) load_p(it + 1);
          if (c + 2 < total && mbar_wait(bar_yz + s, ph, sAbort)) load_o(c + 2);
          // Rows of item it + 1 once the epilogue of item it - 1 is done.
          if (q == 1 && it >= 1 && it + 1 < nit) load_rows(it + 1);
        }
      }
    }
  } else if (warp == MMA_WARP) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t ID_UV = idesc_f16(BM, NC, BF16);
      constexpr uint32_t ID_Y = idesc_f16(BM, D, BF16);
      const uint32_t s0 = smem_u32(sm);
      uint32_t wb0 = s0 + C::OFF_W, wb1 = wb0;  // resident group buffer of the items with parity 0 / 1
      auto issue_y = [&](int x) {  // Y(item) (+)= Z_x B_o[x]
        const int s = x & 1, ix = x / C::NQ, q = x - ix * C::NQ, yb = ix & 1;
        const uint32_t ph = (x >> 1) & 1;
        // Y buffer yb was last read by the epilogue of item ix - 2.
        if (q == 0 && ix >= 2) mbar_wait(bar_epd + (ix & 1), ((ix - 2) >> 1) & 1, sAbort);
        mbar_wait(bar_z + s, ph, sAbort);
        if (!C::RES) mbar_wait(bar_wo + s, ph, sAbort);
        tc_fence_after();
        if (!*sAbort) {
          const uint32_t aZ = s0 + C::OFF_Z + s * C::Z_BYTES;
          const uint32_t aW = C::RES ? ((ix & 1) ? wb1 : wb0) + q * C::IMG_BYTES + C::WUV_BYTES
                                     : s0 + C::OFF_WO + s * C::WO_BYTES;
#pragma unroll
          for (int kk = 0; kk < NC / 16; ++kk)
            umma_f16(tbase + C::T_Y(yb), sdesc_sw128(sw128_kstep(aZ, kk, BM)),
                     sdesc_sw128(sw128_kstep(aW, kk, D)), ID_Y, (q > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(bar_yz + s);
      };
      int c = 0, e = 0;
      for (int it = 0; it < nit; ++it) {
        const bool newgrp = C::RES && it > 0 && qc_of(it) != qc_of(it - 1);
        if (!EARLY && it > 0) {
          // One item buffer: finish the previous item, then hold this item's
          // MMAs until the previous epilogue (warp MMAs) is done.
          issue_y(c - 1);
          mbar_wait(bar_epd + ((it - 1) & 1), ((it - 1) >> 1) & 1, sAbort);
        }
        if (C::RES) {
          if (newgrp) ++e;
          ((it & 1) ? wb1 : wb0) = s0 + C::OFF_W + (e & 1) * C::GRP_BYTES;
          if (it == 0 || newgrp) mbar_wait(bar_wres + (e & 1), (e >> 1) & 1, sAbort);
        }
        mbar_wait(bar_p + it % C::NB, (it / C::NB) & 1, sAbort);
        tc_fence_after();
        const uint32_t aPu = s0 + C::OFF_P + (it % C::NB) * C::PP_BYTES, aPv = aPu + C::P_BYTES;
        for (int q = 0; q < C::NQ; ++q, ++c) {
          const int s = c & 1;
          const uint32_t ph = (c >> 1) & 1;
          if (!C::RES) mbar_wait(bar_wuv + s, ph, sAbort);
          tc_fence_after();
          if (!*sAbort) {
            const uint32_t aBu = C::RES ? ((it & 1) ? wb1 : wb0) + q * C::IMG_BYTES : s0 + C::OFF_WUV + s * C::WUV_BYTES;
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
          if (q == C::NQ - 1) umma_commit(bar_pf + it % C::NB);
          if (c > 0 && (EARLY || q > 0)) {
            issue_y(c - 1);
            // The previous item's last Y was the last reader of its group buffer.
            if (q == 0 && newgrp) umma_commit(bar_wfree + ((e - 1) & 1));
          }
        }
      }
      if (total > 0) issue_y(total - 1);
    }
  } else {
    // ------------------------------------------------ compute warps
    const int g = lane >> 2, t4 = lane & 3;
    uint32_t fo[4];  // A_o as an m16n8k16 A fragment
    load_afrag(amat + 512, false, g, t4, fo);
    // Gate: warp (lq, hw) reads TMEM lanes 32 lq .. +31, columns 32 hw .. +31
    // of a chunk.  Epilogue: the same warp owns tile 2 lq + hw (TMEM lanes
    // 32 lq + 16 hw .. +15) and all D channels.
    const int lq = warp & 3, hw = warp >> 2;
    const int r = lq * 32 + lane, cb = hw * 32;
    const uint32_t trow = tbase + ((uint32_t)(lq * 32) << 16);
    const int tile_e = 2 * lq + hw;
    constexpr int NP = D / 16;  // 16-channel steps of the epilogue
    constexpr int NH = D / 64;  // 64-channel passes
    float* stg = reinterpret_cast<float*>(sm + C::OFF_STG + warp * C::STG_WARP);

    // Channel-group state, reloaded when the group changes (rarely: items
    // are walked group-major).
    int cur_qc = -1, ch0 = 0, sstr = 0;
    bool cont = false;
    float gam[NP][4];  // gamma of channels np 16 + nb 8 + 2 t4 + e at [np][2 nb + e]
    auto set_group = [&](int qc) {
      if (qc == cur_qc) return;
      cur_qc = qc;
      ch0 = p.ch[qc * D];
      const int lay = vec_ok ? contig[qc] : 0;
      cont = layout_stride(lay) == 1;
      sstr = layout_stride(lay) > 1 ? layout_stride(lay) : 0;  // channels ch0 + sstr k
#pragma unroll
      for (int np = 0; np < NP; ++np)
#pragma unroll
        for (int e = 0; e < 4; ++e) gam[np][e] = gg[qc * D + np * 16 + (e >> 1) * 8 + 2 * t4 + (e & 1)];
    };

    // -------- gate: Z_x = silu(U_x) * V_x for chunk x
    auto gate = [&](int cx) {
      const int s = cx & 1;
      const uint32_t ph = (cx >> 1) & 1;
      const int it = cx / C::NQ, q = cx - it * C::NQ;
      mbar_wait(bar_uv + s, ph, sAbort);
      __syncwarp();
      tc_fence_after();
      uint32_t ur[32], vr[32];
      tmem_ld32(trow + C::T_U(s) + cb, ur);
      tmem_ld32(trow + C::T_V(s) + cb, vr);
      tmem_ld_wait();
      if (cx >= 2) mbar_wait(bar_yz + s, ((cx - 2) >> 1) & 1, sAbort);
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
      mbar_arrive(bar_z + s);
    };

    // -------- epilogue state of one item: the output rows of this warp's
    // tile (C-fragment rows g, g + 8), their sample scales, and the residual
    // of the first staged half-pass (requested ahead of use; pad rows read
    // row 0 and are never stored, so no load waits for a comparison).
    int rowf[2];
    float scf[2];
    uint4 xb[2][4];
    const int* sRowsE = nullptr;
    // Residual of half-pass sp (64-channel pass sp >> 1, tile rows 8 (sp & 1)
    // .. +8) in the read-back layout: lane handles row 8 (sp & 1) + ((i * 32 +
    // lane) >> 4), channels 4 (lane & 15) .. +4 of the pass, for i < 4.
    auto xload = [&](int sp, uint4 (&dst)[4]) {
      const int hf = sp >> 1, hr = sp & 1;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int rw = sRowsE[tile_e * 16 + hr * 8 + ((i * 32 + lane) >> 4)];
        const int64_t off = (int64_t)(rw >= 0 ? rw : 0) * p.C + ch0 + hf * 64 + (lane & 15) * 4;
        if constexpr (sizeof(TX) == 2) {
          const uint2 v = __ldg(reinterpret_cast<const uint2*>(x + off));
          dst[i] = make_uint4(v.x, v.y, 0u, 0u);
        } else {
          dst[i] = __ldg(reinterpret_cast<const uint4*>(x + off));
        }
      }
    };
    auto epi_prepare = [&](int it) {
      const int sl = it & 1;
      set_group(qc_of(it));
      mbar_wait(bar_m + sl, (it >> 1) & 1, sAbort);
      if (*sAbort) return;  // the rows never arrived: no load or store may use them
      sRowsE = reinterpret_cast<const int*>(sm + C::OFF_ROWS + sl * C::ROWS_BYTES);
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        rowf[hr] = sRowsE[tile_e * 16 + g + 8 * hr];
        scf[hr] = scale ? scale[(rowf[hr] >= 0 ? rowf[hr] : 0) / p.N] : 1.f;
      }
      if (cont && residual) xload(0, xb[0]);
    };

    // -------- epilogue: delta = A_o Y, gamma, sample scale, residual.  Per
    // 64-channel pass the warp MMA results (C-fragment layout) are scaled by
    // gamma and the row's sample scale, and each half (rows g / g + 8) goes
    // through the warp's f32 staging tile so that 16 lanes write one
    // 128-byte row segment (bf16) with the residual added on the way out.
    auto epilogue = [&](int it) {
      const int yb = it & 1, cl = it * C::NQ + C::NQ - 1;
      mbar_wait(bar_yz + (cl & 1), (cl >> 1) & 1, sAbort);
      if (*sAbort) return;
      __syncwarp();
      tc_fence_after();
      const int* sRows = sRowsE;
      const uint32_t ta = tbase + ((uint32_t)(tile_e * 16) << 16) + C::T_Y(yb);
      uint32_t yv[NP][8];
#pragma unroll
      for (int np = 0; np < NP; ++np) tmem_ld16x256_x2(ta + np * 16, yv[np]);
      tmem_ld_wait();
      const bool res_vec = cont && residual;
#pragma unroll
      for (int hf = 0; hf < NH; ++hf) {
        float cc[4][2][4];  // [16-channel step][channel block nb][C fragment]
#pragma unroll
        for (int n4 = 0; n4 < 4; ++n4) {
          const int np = hf * 4 + n4;
          uint32_t ay[4];
#pragma unroll
          for (int q = 0; q < 4; ++q)
            ay[q] = pack2<BF16>(__uint_as_float(yv[np][2 * q]), __uint_as_float(yv[np][2 * q + 1]));
#pragma unroll
          for (int nb = 0; nb < 2; ++nb) {
            cc[n4][nb][0] = cc[n4][nb][1] = cc[n4][nb][2] = cc[n4][nb][3] = 0.f;
            mma16816<BF16>(cc[n4][nb], fo, movm_trans(ay[2 * nb]), movm_trans(ay[2 * nb + 1]));
          }
        }
        if (sstr) {
          // Strided group: the same staging, then 16 lanes store 16
          // consecutive k of one row (sstr elements apart in the output),
          // reading the residual at the same positions.
#pragma unroll
          for (int hr = 0; hr < 2; ++hr) {
            const float sc = scf[hr];
#pragma unroll
            for (int n4 = 0; n4 < 4; ++n4)
#pragma unroll
              for (int nb = 0; nb < 2; ++nb) {
                const float* gm = gam[hf * 4 + n4] + 2 * nb;
                *reinterpret_cast<float2*>(stg + g * C::ST_LD + n4 * 16 + nb * 8 + 2 * t4) =
                    make_float2(cc[n4][nb][2 * hr] * gm[0] * sc, cc[n4][nb][2 * hr + 1] * gm[1] * sc);
              }
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int r8 = (i * 32 + lane) >> 4;
              const int rw = sRows[tile_e * 16 + hr * 8 + r8];
              const int64_t rowoff = (int64_t)(rw >= 0 ? rw : 0) * p.C + ch0 + (int64_t)sstr * hf * 64;
              float xr[4] = {0.f, 0.f, 0.f, 0.f};
              if (residual) {
#pragma unroll
                for (int m = 0; m < 4; ++m) xr[m] = load_as<float>(x, rowoff + (int64_t)sstr * ((lane & 15) + 16 * m));
              }
              if (rw >= 0) {
#pragma unroll
                for (int m = 0; m < 4; ++m) {
                  const int k = (lane & 15) + 16 * m;
                  out[rowoff + (int64_t)sstr * k] = Elem<TO>::from(stg[r8 * C::ST_LD + k] + xr[m]);
                }
              }
            }
            __syncwarp();  // the staging tile is rewritten by the next half-pass
          }
        } else if (cont) {
#pragma unroll
          for (int hr = 0; hr < 2; ++hr) {
            const int sp = hf * 2 + hr;
            if (res_vec && sp + 1 < 2 * NH) xload(sp + 1, xb[(sp + 1) & 1]);
            const float sc = scf[hr];
#pragma unroll
            for (int n4 = 0; n4 < 4; ++n4)
#pragma unroll
              for (int nb = 0; nb < 2; ++nb) {
                const float* gm = gam[hf * 4 + n4] + 2 * nb;
                *reinterpret_cast<float2*>(stg + g * C::ST_LD + n4 * 16 + nb * 8 + 2 * t4) =
                    make_float2(cc[n4][nb][2 * hr] * gm[0] * sc, cc[n4][nb][2 * hr + 1] * gm[1] * sc);
              }
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int r8 = (i * 32 + lane) >> 4, c4 = (lane & 15) * 4;
              const float4 a = *reinterpret_cast<const float4*>(stg + r8 * C::ST_LD + c4);
              float ov[4] = {a.x, a.y, a.z, a.w};
              if (residual) {
                const uint4 xv = xb[sp & 1][i];
                if constexpr (sizeof(TX) == 2) {
                  const float2 f0 = unpack2<std::is_same_v<TX, __nv_bfloat16>>(xv.x);
                  const float2 f1 = unpack2<std::is_same_v<TX, __nv_bfloat16>>(xv.y);
                  ov[0] += f0.x; ov[1] += f0.y; ov[2] += f1.x; ov[3] += f1.y;
                } else {
                  ov[0] += __uint_as_float(xv.x); ov[1] += __uint_as_float(xv.y);
                  ov[2] += __uint_as_float(xv.z); ov[3] += __uint_as_float(xv.w);
                }
              }
              const int rw = sRows[tile_e * 16 + hr * 8 + r8];
              if (rw >= 0) {
                TO* dst = out + (int64_t)rw * p.C + ch0 + hf * 64 + c4;
                if constexpr (std::is_same_v<TO, float>) {
                  *reinterpret_cast<float4*>(dst) = make_float4(ov[0], ov[1], ov[2], ov[3]);
                } else {
                  constexpr bool OB = std::is_same_v<TO, __nv_bfloat16>;
                  *reinterpret_cast<uint2*>(dst) = make_uint2(pack2<OB>(ov[0], ov[1]), pack2<OB>(ov[2], ov[3]));
                }
              }
            }
            __syncwarp();  // the staging tile is rewritten by the next half-pass
          }
        } else {
          // Channels not one aligned run: element stores (channel list and
          // gamma read through the cache).
          const int* chq = p.ch + cur_qc * D;
          const float* gq = gg + cur_qc * D;
#pragma unroll
          for (int n4 = 0; n4 < 4; ++n4)
#pragma unroll
            for (int nb = 0; nb < 2; ++nb) {
              const int k = (hf * 4 + n4) * 16 + nb * 8 + 2 * t4;
#pragma unroll
              for (int hr = 0; hr < 2; ++hr) {
                const int row = rowf[hr];
                if (row < 0) continue;
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                  const int ch = chq[k + e];
                  if (ch >= p.C) continue;
                  const int64_t off = (int64_t)row * p.C + ch;
                  float dv = cc[n4][nb][2 * hr + e] * gq[k + e] * scf[hr];
                  if (residual) dv += load_as<float>(x, off);
                  out[off] = Elem<TO>::from(dv);
                }
              }
            }
        }
      }
      tc_fence_before();
      mbar_arrive(bar_epd + (it & 1));
    };

    if constexpr (EARLY) {
      if (nit > 0) gate(0);
      for (int it = 0; it < nit; ++it) {
        for (int q = 1; q < C::NQ; ++q) gate(it * C::NQ + q);
        epi_prepare(it);
        if (it + 1 < nit) gate((it + 1) * C::NQ);
        epilogue(it);
      }
    } else {
      for (int it = 0; it < nit; ++it) {
        for (int q = 0; q < C::NQ; ++q) gate(it * C::NQ + q);
        epi_prepare(it);
        epilogue(it);
      }
    }
  }

  __syncwarp();
  __syncthreads();
  report_abort(sAbort, fault);
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
           (uint16_t*)(base + w.amat), (float*)(base + w.gg), (float*)(base + w.nwc),
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
  const bool gather = tcf_covers(a, p);
  TcWs<D> w(p, gather);
  unsigned char* base = (unsigned char*)ws.take(w.total);
  if (!ws.base) return OW_OK;
  int* fault = nullptr;
  OW_RETURN_IF(fault_word(&fault));
  OW_RETURN_IF((tc_prep<D, BF16>(a, p, w, base, st)));
  if (gather) {
    // No pre-pass: its profiling events (if set) bracket nothing.
    profile_mark(OW_PROF_FPACK, false, st);
    profile_mark(OW_PROF_FPACK, true, st);
    return tcf_forward(a, p, base + w.img, (const uint16_t*)(base + w.amat), (const float*)(base + w.gg),
                       (const float*)(base + w.nwc), (const int*)(base + w.contig), st);
  }
  profile_mark(OW_PROF_FPACK, false, st);
  OW_RETURN_IF((tc_pack_forward(a, p, (const uint16_t*)(base + w.amat), (const float*)(base + w.nwc),
                                (const int*)(base + w.contig), base + w.packed, st)));
  profile_mark(OW_PROF_FPACK, true, st);
  const int64_t items = (int64_t)p.Qc * ((p.BQ() + 7) / 8);
  const int grid = (int)std::min<int64_t>(items, device_sm_count());
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
    launch(kern, grid, TC_THREADS, Cfg<D>::SMEM, st, p, (const TX*)a->x,
           (const unsigned char*)(base + w.packed), (const unsigned char*)(base + w.img),
           (const uint16_t*)(base + w.amat), (const float*)(base + w.gg), (const int*)(base + w.contig),
           a->sample_scale, a->residual, (TO*)a->out, vec_ok, fault, wait_probe_ns());
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
  // out_dtype is the forward's output type and the backward's dout type; the
  // sizing call reads it too, so the check never depends on ``out``.
  if (a->out_dtype != c16 && a->out_dtype != OW_DTYPE_F32) return no("out dtype");
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
