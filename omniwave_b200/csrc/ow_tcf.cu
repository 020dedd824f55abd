// Tensor-core BiGEMM forward with TMA row gathers and tcgen05 token mixes
// (sm_100a; bf16/f16 compute; g = 16, d in {64, 128}, rd = 2d; channel
// groups that are runs of d consecutive channels; operator mode, and block
// mode with a 16-bit x: RMSNorm applied to the gathered tile in shared
// memory, the residual added in the epilogue).
//
// Work unit ("item"): one channel group q and an M-block of 128 token rows
// (8 tiles of 16).  Per item (reference.py:147-171, with pack_tiles folded
// into the loads and unpack_tiles into the stores):
//
//   T     = x[rows, q d : q d + d]                  TMA tile::gather4 from x itself (pad rows read the
//                                                   out-of-range fill, 0): no tile is materialised in HBM
//   P^T_t = T_t^T [A_u^T | A_v^T]   per tile t      tcgen05.mma, M = channels, N = 32, K = 16 tokens
//   P_u, P_v -> shared memory                       compute warps (MN-major A operands: lanes = channels)
//   U_c = P_u B_u[:, c],  V_c = P_v B_v[:, c]       tcgen05.mma per 64-feature chunk c, f32 in TMEM
//   Z_c = silu(U_c) V_c                             compute warps
//   Y  += Z_c B_o[c, :]                             tcgen05.mma
//   Y -> shared memory;  Delta^T_t = Y_t^T A_o^T    tcgen05.mma, M = channels, N = 16
//   out[row, q d + c] = Delta[row, c] gamma[c] s_b  compute warps, lanes = consecutive channels
//
// The 16x16 token mixes run on the tensor cores in transposed form: the
// channels fill the M = 128 rows of the MMA, a tile's 16 tokens are K.  At
// d = 64 a mix pairs two tiles to fill M = 128: the T (and Y) images hold
// tile 2j's rows in the first 64-channel atom and tile 2j+1's in the second,
// each beside 16 zero lines, so two K = 16 steps compute both tiles' mixes
// (rows 0-63: tile 2j, rows 64-127: tile 2j+1).
//
// Roles (320 threads): warps 0-7 compute, warp 8 issues every tcgen05.mma
// (one thread) and owns the TMEM allocation, warp 9 issues the TMA gathers
// (all lanes) and the weight copies.  The grid is persistent (one CTA per SM)
// and walks items channel-group-major, so neighbouring CTAs share a group's
// weight images through L2.  Every wait is bounded (ow_sm100.cuh).

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>
#include <type_traits>

#include "ow_common.cuh"
#include "ow_internal.h"
#include "ow_sm100.cuh"

namespace ow {
namespace {

using namespace sm100;

constexpr int BM = 128;                 // token rows per item (8 tiles of 16)
constexpr int NC = 64;                  // rd chunk width
constexpr int NCW = 8;                  // compute warps
constexpr int NCT = NCW * 32;
constexpr int MMA_W = NCW;
constexpr int PROD_W = NCW + 1;          // TMA row gathers
constexpr int WGT_W = NCW + 2;           // weight copies
constexpr int THREADS = (NCW + 3) * 32;
constexpr int TMEM_COLS = 512;
constexpr int ATOM = BM * 128;          // 64 channels x 128 lines, 128-byte swizzled (16 KB)
constexpr int kFaultLayout = 2;         // fault code: a group is not a run of d channels

template <int D>
struct FC {
  static constexpr int RD = 2 * D;
  static constexpr int NQ = RD / NC;             // 64-feature chunks per item
  static constexpr bool PAIR = D == 64;          // token mixes pair two tiles
  static constexpr int NBLK = PAIR ? 4 : 8;      // column blocks of a token mix in TMEM
  static constexpr int T_BYTES = 2 * ATOM;       // T image (d=128: channel halves; d=64: tile parities)
  static constexpr int PI_ATOM = D * 128;        // P image: one 64-token atom of D channel lines
  static constexpr int PI_BYTES = 2 * PI_ATOM;   // P image: 128 tokens
  static constexpr int Z_BYTES = BM * NC * 2;    // one Z chunk (K-major, 128 x 64)
  static constexpr int Y_BYTES = 2 * ATOM;       // Y image (same arrangement as the T image)
  static constexpr int BU_BYTES = NC * D * 2;    // one of B_u / B_v of a chunk image
  static constexpr int WUV_BYTES = 2 * BU_BYTES;
  static constexpr int WO_BYTES = D * NC * 2;
  static constexpr int IMG_BYTES = WUV_BYTES + WO_BYTES;  // chunk image [B_u | B_v | B_o] (prep kernel)
  // Shared memory.  d = 64: T, P images, Z, Y image and the resident weights
  // of one channel group each have their own region (the T and Y images
  // keep their zero lines).  d = 128: the Y image overwrites the Z buffers
  // once the last Y MMA has read them, and the weights stream per chunk,
  // [B_u | B_v] through two stages and B_o through one.
  // d = 64 double-buffers the T image, so the next item's rows land (and, in
  // block mode, are normalised) while this item's image is still in use.
  static constexpr int NTB = PAIR ? 2 : 1;
  static constexpr int OFF_T = 0;
  __host__ __device__ static constexpr int T_OFF(int b) { return OFF_T + b * T_BYTES; }
  static constexpr int OFF_PU = NTB * T_BYTES;
  static constexpr int OFF_PV = OFF_PU + PI_BYTES;
  static constexpr int R_END = OFF_PV + PI_BYTES;
  static constexpr int OFF_Z = R_END;
  static constexpr int OFF_Y = PAIR ? OFF_Z + 2 * Z_BYTES : OFF_Z;
  static constexpr int OFF_W = PAIR ? OFF_Y + Y_BYTES : OFF_Z + 2 * Z_BYTES;
  static constexpr int OFF_WUV = OFF_W;                               // d = 128: 2 x [B_u | B_v]
  static constexpr int OFF_WO = OFF_WUV + 2 * WUV_BYTES;              // d = 128: B_o
  static constexpr int W_END = PAIR ? OFF_W + NQ * IMG_BYTES : OFF_WO + WO_BYTES;
  static constexpr int OFF_BUV = W_END;                               // mix B images (K-major, SW128)
  static constexpr int OFF_BO = OFF_BUV + 32 * 128;
  static constexpr int OFF_ROWS = OFF_BO + 16 * 128;                  // 2 x output row of each token row
  static constexpr int OFF_RS = OFF_ROWS + 2 * BM * 4;                // block mode: 2 x rstd of each token row
  static constexpr int OFF_BAR = OFF_RS + 2 * BM * 4;
  static constexpr int NBAR = 24;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;
  // TMEM columns.
  static constexpr int T_PM = 0;                                 // P^T blocks (32 columns each)
  __host__ __device__ static constexpr int T_U(int s) { return 128 * s; }
  __host__ __device__ static constexpr int T_V(int s) { return 128 * s + 64; }
  static constexpr int T_Y = 256;
  static constexpr int T_DT = 256 + D;                           // Delta^T blocks (16 columns each)
  static_assert(T_PM + 32 * NBLK <= 256 && T_DT + 16 * NBLK <= TMEM_COLS, "TMEM budget");
  static_assert(PAIR || Y_BYTES <= 2 * Z_BYTES, "d = 128: the Y image fits where the Z buffers go");
  static_assert(SMEM <= 232448, "shared memory budget");
};

// Instruction descriptor with the A operand MN-major (B K-major).
__host__ __device__ constexpr uint32_t idesc_amn(int M, int N, bool bf16) { return idesc_f16(M, N, bf16) | (1u << 15); }

// Descriptor of an SW128 operand read MN-major: 64-element MN atoms ``lbo``
// bytes apart, 8-line K groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sdesc_mn(uint32_t addr, uint32_t lbo) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Byte offset of 16-byte chunk ``kc`` (0..7) of line ``ln`` in a 128-byte
// swizzled region whose 8-line groups are 1024 bytes apart.
__device__ __forceinline__ uint32_t line_chunk(int ln, int kc) {
  return (uint32_t)((ln >> 3) * 1024 + (ln & 7) * 128 + ((kc ^ (ln & 7)) << 4));
}

// TMA: four rows (row0..row3 of a 2-D tensor map), ``col`` .. col + box - 1
// each, into consecutive 128-byte lines at ``dst``; completes on ``bar``.
__device__ __forceinline__ void tma_gather4(void* dst, const CUtensorMap* map, int col, int r0, int r1, int r2,
                                            int r3, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(col), "r"(r0), "r"(r1), "r"(r2), "r"(r3), "r"(smem_u32(bar))
      : "memory");
}

// Line of token row r (tile r / 16, row r % 16) in a T or Y image, and the
// 64-channel atom that holds channel column ``c``.  d = 128: atom = c / 64,
// line = r.  d = 64 (paired tiles): atom = tile parity, line = 32 (tile / 2)
// + 16 (tile % 2) + r % 16.
template <int D>
__device__ __forceinline__ uint32_t img_off(int r, int c) {
  if constexpr (D == 64) {
    const int t = r >> 4;
    return (uint32_t)((t & 1) * ATOM) + line_chunk(32 * (t >> 1) + 16 * (t & 1) + (r & 15), c >> 3);
  } else {
    return (uint32_t)((c >> 6) * ATOM) + line_chunk(r, (c & 63) >> 3);
  }
}

// Block mode (fused OmniWeaveBlock, reference block.py:80-108): the gathered
// tile is RMS-normalised in shared memory, T = round(round(x rstd) nw) in x's
// dtype, and the epilogue adds the residual, out = x + scale_b Delta.
struct BlockArgs {
  const float* rstd;  // [B N] per token row
  const float* nw;    // [C] norm weight (f32 copy)
  const void* x;      // the residual (x itself, in the 16-bit compute type)
};

template <int D, bool BF16, typename TO, bool RES>
__global__ void __launch_bounds__(THREADS, 1)
tcf_kernel(const __grid_constant__ CUtensorMap xmap, Prob p, const unsigned char* __restrict__ img,
           const uint16_t* __restrict__ amat, const float* __restrict__ gg, const int* __restrict__ layout,
           const float* __restrict__ scale, TO* __restrict__ out, BlockArgs blk, int* fault, uint32_t probe_ns) {
  using C = FC<D>;
  using T16 = std::conditional_t<BF16, __nv_bfloat16, __half>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + C::OFF_BAR);
  // Per T buffer b (selects, not arrays: no local memory):
  auto bar_t = [&](int b) { return b ? bars + 21 : bars + 0; };       // image gathered (tx)
  uint64_t* bar_pm = bars + 1;      // P^T mix done (commit)
  uint64_t* bar_p = bars + 2;       // P images written (compute)
  uint64_t* bar_uv = bars + 3;      // [2] U/V of TMEM buffer s computed (commit)
  uint64_t* bar_z = bars + 5;       // [2] Z_s written, TMEM buffer s read (compute)
  uint64_t* bar_yz = bars + 7;      // [2] Y MMA of Z buffer s done (commit)
  uint64_t* bar_wuv = bars + 9;     // [2] d = 128: [B_u | B_v] stage loaded (tx); d = 64: group loaded (tx)
  uint64_t* bar_wo = bars + 11;     // d = 128: B_o stage loaded (tx)
  uint64_t* bar_wfree = bars + 13;  // d = 64: the resident group is no longer read (commit)
  auto bar_rfree = [&](int b) { return b ? bars + 22 : bars + 14; };  // image read: it may take the next item (commit)
  uint64_t* bar_y = bars + 15;      // Y of the item complete (commit)
  uint64_t* bar_yi = bars + 16;     // Y image written (compute)
  uint64_t* bar_dt = bars + 17;     // Delta^T mix done (commit)
  uint64_t* bar_epd = bars + 18;    // epilogue done: Delta^T columns read (compute)
  uint64_t* bar_probe = bars + 19;  // wait-timeout self-check: nothing arrives on it
  auto bar_tn = [&](int b) { return b ? bars + 23 : bars + 20; };     // block mode: image normalised (producer, all lanes)
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(bars + C::NBAR);
  volatile int* sAbort = reinterpret_cast<volatile int*>(sTmem + 1);
  int* sRows = reinterpret_cast<int*>(sm + C::OFF_ROWS);
  float* sRs = reinterpret_cast<float*>(sm + C::OFF_RS);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t BQ = (int64_t)p.B * p.Qs;
  const int nMB = (int)((BQ + 7) / 8);
  const int64_t items = (int64_t)p.Qc * nMB;
  const int nit = items > blockIdx.x ? (int)((items - 1 - blockIdx.x) / gridDim.x + 1) : 0;
  const int oob = p.B * p.N;  // a row coordinate past the tensor: TMA fills zeros
  auto item_of = [&](int it) { return (int64_t)blockIdx.x + (int64_t)it * gridDim.x; };
  auto qc_of = [&](int it) { return (int)(item_of(it) / nMB); };
  auto mb_of = [&](int it) { return (int)(item_of(it) - (int64_t)qc_of(it) * nMB); };
  // Output row (b N + token) of row r of M-block mb, or -1 for a pad row.
  // (B Q_s < 2^31 is checked on the host, so 32-bit arithmetic suffices.)
  auto row_of = [&](int mb, int r) -> int {
    const int tt = mb * 8 + (r >> 4);
    if (tt >= (int)BQ) return -1;
    const int b = tt / p.Qs;
    const int tok = p.tok[(tt - b * p.Qs) * 16 + (r & 15)];
    return tok < p.N ? b * p.N + tok : -1;
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::NBAR; ++i) {
      const bool comp = bars + i == bar_p || bars + i == bar_yi || bars + i == bar_epd || bars + i == bar_z ||
                        bars + i == bar_z + 1;
      mbar_init(bars + i, comp ? NCT : (bars + i == bar_tn(0) || bars + i == bar_tn(1) ? 32 : 1));
    }
    *sAbort = 0;
    // The kernel covers channel groups that are one aligned run of d channels.
    for (int q = 0; q < p.Qc; ++q)
      if (layout_stride(layout[q]) != 1) {
        atomicOr(fault, kFaultLayout);
        *sAbort = 1;
      }
    fence_mbar_init();
    wait_probe(bar_probe, sAbort, probe_ns);
  }
  // Mix B operands (K-major, 128-byte swizzled, K = 16): rows 0-15 A_u,
  // rows 16-31 A_v (BUV, B[k][n] = A[n][k]), and A_o (BO); the 16-element
  // rows occupy chunks 0-1 of each 128-byte line.  At d = 64 the T and Y
  // images' zero lines are written once here.
  if (warp < NCW) {
    const int tid = threadIdx.x;
    for (int i = tid; i < 48 * 16; i += NCT) {
      const int n = i >> 4, k = i & 15;
      const uint16_t v = n < 16 ? amat[n * 16 + k] : (n < 32 ? amat[256 + (n - 16) * 16 + k] : amat[512 + (n - 32) * 16 + k]);
      const uint32_t base = n < 32 ? C::OFF_BUV : C::OFF_BO;
      const int nn = n < 32 ? n : n - 32;
      *reinterpret_cast<uint16_t*>(sm + base + line_chunk(nn, k >> 3) + (k & 7) * 2) = v;
    }
    if constexpr (C::PAIR) {
      // Zero lines: atom 0 lines 32j + 16 .. +15, atom 1 lines 32j .. +15.
      for (int i = tid; i < 4 * 16 * 2 * 8; i += NCT) {
        const int kc = i & 7, ln16 = (i >> 3) & 15, j = (i >> 7) & 3, a = i >> 9;
        const int ln = 32 * j + (a == 0 ? 16 : 0) + ln16;
        const uint4 z = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int b = 0; b < C::NTB; ++b) *reinterpret_cast<uint4*>(sm + C::T_OFF(b) + a * ATOM + line_chunk(ln, kc)) = z;
        *reinterpret_cast<uint4*>(sm + C::OFF_Y + a * ATOM + line_chunk(ln, kc)) = z;
      }
    }
    fence_proxy_async_smem();
  }
  if (warp == MMA_W) tmem_alloc(sTmem, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *sTmem;

  // Block mode: T <- round(round(T rstd[row]) nw[channel]) in place once the
  // rows of item it have landed (pad rows are zero and have rstd 0), by one
  // warp with all lanes: the weight warp at d = 64 (its weights are
  // resident), the producer at d = 128.  The item's mix waits on bar_tn.
  // Lane l always handles 16-byte chunk l % (D / 8) of its rows, so its eight
  // norm-weight values are loaded once per item.
  auto normalize = [&](int it) -> bool {
    const int tb = it % C::NTB, tk = it / C::NTB;
    constexpr int CPR = D / 8;  // 16-byte chunks per row
    const int c = (lane % CPR) * 8;
    const float* nwq = blk.nw + p.ch[qc_of(it) * D] + c;
    const float4 n0 = __ldg(reinterpret_cast<const float4*>(nwq));
    const float4 n1 = __ldg(reinterpret_cast<const float4*>(nwq + 4));
    const float nv[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
    if (!mbar_wait(bar_t(tb), tk & 1, sAbort)) return false;
    const float* srs = sRs + (it & 1) * BM;
#pragma unroll 4
    for (int row = lane / CPR; row < BM; row += 32 / CPR) {
      const float rs = srs[row];
      uint4* ptr = reinterpret_cast<uint4*>(sm + C::T_OFF(tb) + img_off<D>(row, c));
      uint4 w = *ptr;
      uint32_t* wp = &w.x;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        // x is in the compute type here, so both roundings go through it.
        const float2 f = unpack2<BF16>(wp[e]);
        const float2 t = unpack2<BF16>(pack2<BF16>(f.x * rs, f.y * rs));
        wp[e] = pack2<BF16>(t.x * nv[2 * e], t.y * nv[2 * e + 1]);
      }
      *ptr = w;
    }
    fence_proxy_async_smem();
    mbar_arrive(bar_tn(tb));
    return true;
  };

  if (*sAbort) {
    // The wait-timeout self-check ran out, or a group is not a channel run:
    // nothing is issued.
  } else if (warp == PROD_W) {
    // ------------------------------------------------ producer: TMA row gathers
    for (int it = 0; it < nit && !*sAbort; ++it) {
      const int qc = qc_of(it), mb = mb_of(it);
      // Rows (and, in block mode, their RMS factors) are fetched before the
      // wait for the T region, so their loads overlap it.
      int rw[4];
      float rsv[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int r = row_of(mb, 4 * lane + j);
        rw[j] = r >= 0 ? r : oob;
        if constexpr (RES) rsv[j] = r >= 0 ? blk.rstd[r] : 0.f;
      }
      // T buffer tb is free once the mix of its previous item has read it.
      const int tb = it % C::NTB, tk = it / C::NTB;
      if (it >= C::NTB && !mbar_wait(bar_rfree(tb), (tk - 1) & 1, sAbort)) break;
      if constexpr (RES) {
        // Published to the compute warps by the arrive below (release) and
        // the completion of bar_t (acquire).
#pragma unroll
        for (int j = 0; j < 4; ++j) sRs[(it & 1) * BM + 4 * lane + j] = rsv[j];
        __syncwarp();
      }
      if (lane == 0) mbar_arrive_expect_tx(bar_t(tb), BM * D * 2);
      __syncwarp();
      const int ch0 = p.ch[qc * D];  // first channel of the group's run
      if constexpr (C::PAIR) {
        const int t = lane >> 2;
        const uint32_t dst = C::T_OFF(tb) + (t & 1) * ATOM + (32 * (t >> 1) + 16 * (t & 1) + 4 * (lane & 3)) * 128;
        tma_gather4(sm + dst, &xmap, ch0, rw[0], rw[1], rw[2], rw[3], bar_t(tb));
      } else {
#pragma unroll
        for (int a = 0; a < 2; ++a)
          tma_gather4(sm + C::T_OFF(tb) + a * ATOM + 4 * lane * 128, &xmap, ch0 + 64 * a, rw[0], rw[1], rw[2],
                      rw[3], bar_t(tb));
      }
      if constexpr (RES && !C::PAIR) {
        if (!normalize(it)) break;
      }
    }
  } else if (warp == WGT_W) {
    // ------------------------------------------------ weight copies
    if constexpr (C::PAIR) {
      // d = 64: the group's weights, resident, reloaded when the group
      // changes (lane 0); in block mode the warp also normalises each item.
      int wq = -1, ge = 0;  // resident group and number of group loads
      for (int it = 0; it < nit && !*sAbort; ++it) {
        const int qc = qc_of(it);
        const bool newg = qc != wq;
        bool ok = true;
        if (lane == 0 && newg) {
          if (ge > 0 && !mbar_wait(bar_wfree, (ge - 1) & 1, sAbort)) ok = false;
          if (ok) {
            mbar_arrive_expect_tx(bar_wuv, C::NQ * C::IMG_BYTES);
            bulk_g2s(sm + C::OFF_W, img + (int64_t)qc * C::NQ * C::IMG_BYTES, C::NQ * C::IMG_BYTES, bar_wuv);
          }
        }
        if (newg) {
          wq = qc;
          ++ge;
        }
        if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
        if constexpr (RES) {
          if (!normalize(it)) break;
        }
      }
    } else if (lane == 0) {
      if constexpr (!C::PAIR) {
        // [B_u | B_v] of chunk c into stage c & 1 once U/V(c - 2) is done,
        // two chunks ahead; B_o into its single stage once Y(c - 1) is done.
        const int total = nit * C::NQ;
        auto src_of = [&](int c) {
          return img + ((int64_t)qc_of(c / C::NQ) * C::NQ + c % C::NQ) * C::IMG_BYTES;
        };
        auto load_uv = [&](int c) {
          mbar_arrive_expect_tx(bar_wuv + (c & 1), C::WUV_BYTES);
          bulk_g2s(sm + C::OFF_WUV + (c & 1) * C::WUV_BYTES, src_of(c), C::WUV_BYTES, bar_wuv + (c & 1));
        };
        for (int c = 0; c < 2 && c < total; ++c) load_uv(c);
        for (int c = 0; c < total && !*sAbort; ++c) {
          if (c >= 1 && !mbar_wait(bar_yz + ((c - 1) & 1), ((c - 1) >> 1) & 1, sAbort)) break;
          mbar_arrive_expect_tx(bar_wo, C::WO_BYTES);
          bulk_g2s(sm + C::OFF_WO, src_of(c) + C::WUV_BYTES, C::WO_BYTES, bar_wo);
          if (c + 2 < total) {
            if (!mbar_wait(bar_uv + (c & 1), (c >> 1) & 1, sAbort)) break;
            load_uv(c + 2);
          }
        }
      }
    }
  } else if (warp == MMA_W) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t ID_MUV = idesc_amn(BM, 32, BF16);
      constexpr uint32_t ID_MO = idesc_amn(BM, 16, BF16);
      constexpr uint32_t ID_UV = idesc_amn(BM, NC, BF16);
      constexpr uint32_t ID_Y = idesc_f16(BM, D, BF16);
      const uint32_t s0 = smem_u32(sm);
      const uint64_t dBUV = sdesc_sw128(s0 + C::OFF_BUV), dBO = sdesc_sw128(s0 + C::OFF_BO);
      int wq = -1, ge = 0;
      // Token mix of an image (T or Y) into TMEM column blocks of width nb.
      auto mix = [&](uint32_t img_addr, uint32_t tcol, int nb, uint64_t bdesc, uint32_t id) {
        for (int blk = 0; blk < C::NBLK; ++blk) {
          if constexpr (C::PAIR) {
            for (int k2 = 0; k2 < 2; ++k2)
              umma_f16(tbase + tcol + nb * blk, sdesc_mn(img_addr + (32 * blk + 16 * k2) * 128, ATOM), bdesc, id,
                       k2 ? 1u : 0u);
          } else {
            umma_f16(tbase + tcol + nb * blk, sdesc_mn(img_addr + blk * 2048, ATOM), bdesc, id, 0u);
          }
        }
      };
      // The mix of item it + 1 goes between the chunks of item it and its
      // Delta mix, so the compute warps turn it into P images while this
      // item's Delta mix runs, and the next item's first U/V chunks run
      // while they store this item's outputs.
      auto item_mix = [&](int it) {
        const int tb = it % C::NTB, tk = it / C::NTB;
        mbar_wait(RES ? bar_tn(tb) : bar_t(tb), tk & 1, sAbort);
        tc_fence_after();
        if (!*sAbort) mix(s0 + C::T_OFF(tb), C::T_PM, 32, dBUV, ID_MUV);
        umma_commit(bar_pm);
        umma_commit(bar_rfree(tb));  // the T image is read
      };
      if (nit > 0) item_mix(0);
      for (int it = 0; it < nit && !*sAbort; ++it) {
        const int qc = qc_of(it);
        const bool newgrp = qc != wq;
        const int c0 = it * C::NQ;
        if (C::PAIR && newgrp) {
          mbar_wait(bar_wuv, ge & 1, sAbort);
          wq = qc;
          ++ge;
        }
        mbar_wait(bar_p, it & 1, sAbort);
        tc_fence_after();
        auto wuv = [&](int c) -> uint32_t {
          return C::PAIR ? s0 + C::OFF_W + (c - c0) * C::IMG_BYTES : s0 + C::OFF_WUV + (c & 1) * C::WUV_BYTES;
        };
        auto wo = [&](int c) -> uint32_t {
          return C::PAIR ? s0 + C::OFF_W + (c - c0) * C::IMG_BYTES + C::WUV_BYTES : s0 + C::OFF_WO;
        };
        auto issue_y = [&](int c) {  // Y (+)= Z_c B_o[c]
          const int s = c & 1;
          mbar_wait(bar_z + s, (c >> 1) & 1, sAbort);
          if (!C::PAIR) mbar_wait(bar_wo, c & 1, sAbort);
          tc_fence_after();
          if (!*sAbort) {
            const uint32_t aZ = s0 + C::OFF_Z + s * C::Z_BYTES, aW = wo(c);
#pragma unroll
            for (int kk = 0; kk < NC / 16; ++kk)
              umma_f16(tbase + C::T_Y, sdesc_sw128(sw128_kstep(aZ, kk, BM)), sdesc_sw128(sw128_kstep(aW, kk, D)), ID_Y,
                       (c > c0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(bar_yz + s);
        };
        for (int q = 0; q < C::NQ; ++q) {
          const int c = c0 + q, s = c & 1;
          // TMEM buffer s was last read by the gate of chunk c - 2.
          if (c >= 2) mbar_wait(bar_z + s, ((c - 2) >> 1) & 1, sAbort);
          if (!C::PAIR) mbar_wait(bar_wuv + s, (c >> 1) & 1, sAbort);
          tc_fence_after();
          if (!*sAbort) {
            const uint32_t aBu = wuv(c), aBv = aBu + C::BU_BYTES;
            const uint32_t aPu = s0 + C::OFF_PU, aPv = s0 + C::OFF_PV;
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              umma_f16(tbase + C::T_U(s), sdesc_mn(aPu + kk * 2048, C::PI_ATOM), sdesc_sw128(sw128_kstep(aBu, kk, NC)),
                       ID_UV, kk > 0 ? 1u : 0u);
              umma_f16(tbase + C::T_V(s), sdesc_mn(aPv + kk * 2048, C::PI_ATOM), sdesc_sw128(sw128_kstep(aBv, kk, NC)),
                       ID_UV, kk > 0 ? 1u : 0u);
            }
          }
          umma_commit(bar_uv + s);
          if (q > 0) issue_y(c - 1);
        }
        issue_y(c0 + C::NQ - 1);  // waits for the item's last gate: TMEM columns 0-255 are free
        umma_commit(bar_y);
        if (C::PAIR && (it + 1 == nit || qc_of(it + 1) != qc)) umma_commit(bar_wfree);
        if (it + 1 < nit) item_mix(it + 1);
        // Delta^T = Y^T A_o^T once the Y image is written and the previous
        // epilogue has read its Delta^T columns.
        mbar_wait(bar_yi, it & 1, sAbort);
        if (it >= 1) mbar_wait(bar_epd, (it - 1) & 1, sAbort);
        tc_fence_after();
        if (!*sAbort) mix(s0 + C::OFF_Y, C::T_DT, 16, dBO, ID_MO);
        umma_commit(bar_dt);
      }
    }
  } else {
    // ------------------------------------------------ compute warps
    const int tid = threadIdx.x;
    const int quad = warp & 3, half = warp >> 2;
    const uint32_t tq = tbase + ((uint32_t)(quad * 32) << 16);  // this warp's TMEM lanes
    const int r = quad * 32 + lane;                               // token row (gate, Y image) or lane
    // Channel and tile parity of this thread's TMEM lane in a mix result.
    const int mc = C::PAIR ? (r & 63) : r;
    const int mpar = C::PAIR ? (r >> 6) : 0;
    // ---- output rows of item it and its P images from P^T (lanes =
    // channels).  Two row buffers: the other may still be read by a warp
    // finishing the previous epilogue; the barrier publishes the rows.
    // Output row of token row tid of the next item: the route-table load is
    // issued an item ahead (from a clamped index, so nothing waits for it)
    // and the row is formed when the item's P images are built.
    int ntok = 0, nb = 0, nvalid = 0;
    auto row_issue = [&](int it) {
      const int tt = mb_of(it) * 8 + (tid >> 4);
      nvalid = tt < (int)BQ;
      const int ttc = nvalid ? tt : 0;
      nb = ttc / p.Qs;
      ntok = p.tok[(ttc - nb * p.Qs) * 16 + (tid & 15)];
    };
    auto pconv = [&](int it) {
      int* rows = sRows + (it & 1) * BM;
      if (it == 0 && tid < BM) row_issue(0);
      if (tid < BM) rows[tid] = nvalid && ntok < p.N ? nb * p.N + ntok : -1;
      asm volatile("bar.sync 1, %0;" ::"n"(NCT) : "memory");
      mbar_wait(bar_pm, it & 1, sAbort);
      __syncwarp();
      tc_fence_after();
#pragma unroll
      for (int bb = 0; bb < C::NBLK / 2; ++bb) {
        const int blk = half * (C::NBLK / 2) + bb;
        const int t = C::PAIR ? 2 * blk + mpar : blk;  // tile of this lane's column block
        uint32_t v[32];
        tmem_ld32(tq + C::T_PM + 32 * blk, v);
        tmem_ld_wait();
        // tokens 16 t .. 16 t + 15: atom t / 4, chunks 2 (t % 4) and 2 (t % 4) + 1 of line mc
#pragma unroll
        for (int uv = 0; uv < 2; ++uv) {
          unsigned char* base = sm + (uv ? C::OFF_PV : C::OFF_PU) + (t >> 2) * C::PI_ATOM;
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const uint32_t* e = v + 16 * uv + 8 * j;
            uint4 w;
            w.x = pack2<BF16>(__uint_as_float(e[0]), __uint_as_float(e[1]));
            w.y = pack2<BF16>(__uint_as_float(e[2]), __uint_as_float(e[3]));
            w.z = pack2<BF16>(__uint_as_float(e[4]), __uint_as_float(e[5]));
            w.w = pack2<BF16>(__uint_as_float(e[6]), __uint_as_float(e[7]));
            *reinterpret_cast<uint4*>(base + line_chunk(mc, 2 * (t & 3) + j)) = w;
          }
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(bar_p);
    };
    // ---- gates: Z_c = silu(U_c) V_c (lanes = tokens)
    auto gates = [&](int it) {
      const int c0 = it * C::NQ;
      for (int q = 0; q < C::NQ; ++q) {
        const int c = c0 + q, s = c & 1;
        mbar_wait(bar_uv + s, (c >> 1) & 1, sAbort);
        __syncwarp();
        tc_fence_after();
        uint32_t ur[32], vr[32];
        tmem_ld32(tq + C::T_U(s) + 32 * half, ur);
        tmem_ld32(tq + C::T_V(s) + 32 * half, vr);
        tmem_ld_wait();
        if (c >= 2) mbar_wait(bar_yz + s, ((c - 2) >> 1) & 1, sAbort);  // Z buffer s read by Y(c - 2)
        unsigned char* Zs = sm + C::OFF_Z + s * C::Z_BYTES;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          uint4 w;
          uint32_t* wp = &w.x;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int i0 = jj * 8 + 2 * e;
            const uint32_t u2 = pack2<BF16>(__uint_as_float(ur[i0]), __uint_as_float(ur[i0 + 1]));
            const uint32_t v2 = pack2<BF16>(__uint_as_float(vr[i0]), __uint_as_float(vr[i0 + 1]));
            wp[e] = silu_mul2<BF16>(u2, v2);
          }
          *reinterpret_cast<uint4*>(Zs + sw128_off(r, 32 * half + jj * 8, BM)) = w;
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(bar_z + s);
      }
    };
    // ---- Y image (lanes = tokens): channels [half D / 2, (half + 1) D / 2)
    auto yimg = [&](int it) {
      mbar_wait(bar_y, it & 1, sAbort);
      __syncwarp();
      tc_fence_after();
#pragma unroll
      for (int cb = 0; cb < D / 64; ++cb) {
        const int cbase = half * (D / 2) + 32 * cb;
        uint32_t v[32];
        tmem_ld32(tq + C::T_Y + cbase, v);
        tmem_ld_wait();
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const uint32_t* e = v + 8 * m;
          uint4 w;
          w.x = pack2<BF16>(__uint_as_float(e[0]), __uint_as_float(e[1]));
          w.y = pack2<BF16>(__uint_as_float(e[2]), __uint_as_float(e[3]));
          w.z = pack2<BF16>(__uint_as_float(e[4]), __uint_as_float(e[5]));
          w.w = pack2<BF16>(__uint_as_float(e[6]), __uint_as_float(e[7]));
          *reinterpret_cast<uint4*>(sm + C::OFF_Y + img_off<D>(r, cbase + 8 * m)) = w;
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(bar_yi);
    };
    // ---- epilogue: out[row, c0 + c] = Delta[row, c] gamma[c] s_b.  Delta^T
    // arrives with lanes = channels; the tile goes through shared memory (the
    // Z region, free until the next item's gates) so that the global stores
    // are whole row segments (D channels per row, 16 bytes per lane).  f32
    // outputs at d = 128 take two passes of 64 tokens.
    auto epilogue = [&](int it) {
      const int qc = qc_of(it);
      const int* rows = sRows + (it & 1) * BM;
      const int c0ch = p.ch[qc * D];
      // Block mode stages f32 so the residual add rounds once.
      using TS = std::conditional_t<RES, float, TO>;
      constexpr int STG_ROWS = (BM * D * (int)sizeof(TS) <= 2 * C::Z_BYTES) ? BM : BM / 2;
      constexpr int NPASS = BM / STG_ROWS;
      // Block mode: the residual x of every unit this thread stores (four
      // channels each; rows < 0 load row 0 and store nothing), loaded before
      // the wait for Delta so the loads overlap it.
      constexpr int RVPR = D / 4;
      constexpr int RNU = RES ? STG_ROWS * RVPR / NCT : 1;
      static_assert(!RES || STG_ROWS * RVPR % NCT == 0, "whole units per thread");
      uint2 xv[NPASS][RNU];
      if constexpr (RES) {
        const T16* xr = reinterpret_cast<const T16*>(blk.x);
#pragma unroll
        for (int pass = 0; pass < NPASS; ++pass)
#pragma unroll
          for (int j = 0; j < RNU; ++j) {
            const int u = tid + j * NCT, rl = u / RVPR, vi = u - rl * RVPR;
            const int rw = rows[pass * STG_ROWS + rl];
            xv[pass][j] = __ldg(reinterpret_cast<const uint2*>(xr + (int64_t)(rw >= 0 ? rw : 0) * p.C + c0ch + vi * 4));
          }
      }
      mbar_wait(bar_dt, it & 1, sAbort);
      __syncwarp();
      tc_fence_after();
      if (*sAbort) return;
      const float gm = gg[(int64_t)qc * D + mc];
      constexpr int NCOL = C::PAIR ? 32 : 64;  // Delta^T columns of this warp half
      TS* stg = reinterpret_cast<TS*>(sm + C::OFF_Z);  // [STG_ROWS][D]
      uint32_t v[NCOL];
#pragma unroll
      for (int cc = 0; cc < NCOL; cc += 32) tmem_ld32(tq + C::T_DT + NCOL * half + cc, *reinterpret_cast<uint32_t(*)[32]>(v + cc));
      tmem_ld_wait();
#pragma unroll 1
      for (int pass = 0; pass < NPASS; ++pass) {
        // Delta^T column k of this thread holds token tok(k) of channel mc.
        // The per-sample scale (block mode) is a separate loop: its row ->
        // sample division must not run when there is no scale.
        auto tok_of = [&](int k) {
          const int col = NCOL * half + k;  // block col / 16, token col % 16
          const int t = C::PAIR ? 2 * (col >> 4) + mpar : (col >> 4);
          return 16 * t + (col & 15);
        };
        if (scale) {
#pragma unroll
          for (int k = 0; k < NCOL; ++k) {
            const int tok = tok_of(k);
            if (tok / STG_ROWS == pass) {
              const int rw = rows[tok];
              const float sc = rw >= 0 ? scale[rw / p.N] : 0.f;
              stg[(tok % STG_ROWS) * D + mc] = Elem<TS>::from(__uint_as_float(v[k]) * gm * sc);
            }
          }
        } else {
#pragma unroll
          for (int k = 0; k < NCOL; ++k) {
            const int tok = tok_of(k);
            if (tok / STG_ROWS == pass) stg[(tok % STG_ROWS) * D + mc] = Elem<TS>::from(__uint_as_float(v[k]) * gm);
          }
        }
        asm volatile("bar.sync 1, %0;" ::"n"(NCT) : "memory");
        if constexpr (RES) {
          // out = x + staged, four channels per unit.
#pragma unroll
          for (int j = 0; j < RNU; ++j) {
            const int u = tid + j * NCT, rl = u / RVPR, vi = u - rl * RVPR;
            const int rw = rows[pass * STG_ROWS + rl];
            if (rw >= 0) {
              const float4 sv = *reinterpret_cast<const float4*>(stg + rl * D + vi * 4);
              const uint2 xw = pass == 0 ? xv[0][j] : xv[NPASS - 1][j];
              const float2 x0 = unpack2<BF16>(xw.x), x1 = unpack2<BF16>(xw.y);
              TO* o = out + (int64_t)rw * p.C + c0ch + vi * 4;
              if constexpr (sizeof(TO) == 2) {
                *reinterpret_cast<uint2*>(o) = make_uint2(pack2<BF16>(x0.x + sv.x, x0.y + sv.y),
                                                          pack2<BF16>(x1.x + sv.z, x1.y + sv.w));
              } else {
                *reinterpret_cast<float4*>(o) = make_float4(x0.x + sv.x, x0.y + sv.y, x1.x + sv.z, x1.y + sv.w);
              }
            }
          }
        } else {
          // Row stores: 16 bytes per thread, consecutive threads along a row.
          constexpr int VPR = D * (int)sizeof(TO) / 16;  // 16-byte vectors per row segment
          for (int u = tid; u < STG_ROWS * VPR; u += NCT) {
            const int rl = u / VPR, vi = u - rl * VPR;
            const int rw = rows[pass * STG_ROWS + rl];
            if (rw >= 0) {
              const uint4 val = *reinterpret_cast<const uint4*>(stg + rl * D + vi * (16 / (int)sizeof(TO)));
              *reinterpret_cast<uint4*>(out + (int64_t)rw * p.C + c0ch + vi * (16 / (int)sizeof(TO))) = val;
            }
          }
        }
        asm volatile("bar.sync 1, %0;" ::"n"(NCT) : "memory");  // staging reused by the next pass / the gates
      }
      tc_fence_before();
      mbar_arrive(bar_epd);
    };
    // Order: gates(it), Y image(it), P images(it + 1), epilogue(it) -- the
    // tensor pipe runs the Delta mix of it and the first U/V chunks of it + 1
    // while the epilogue stores.
    if (nit > 0) pconv(0);
    for (int it = 0; it < nit && !*sAbort; ++it) {
      // The next item's row indices: the table load overlaps the gates.
      if (tid < BM && it + 1 < nit) row_issue(it + 1);
      gates(it);
      yimg(it);
      if (it + 1 < nit) pconv(it + 1);
      epilogue(it);
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
  if (warp == MMA_W) {
    tc_fence_after();
    tmem_dealloc(tbase, TMEM_COLS);
  }
}

// 2-D tensor map of x viewed as [B N rows, C channels] (16-bit), box of 64
// channels x 1 row, 128-byte swizzle: the row-gather source of the kernel.
int make_xmap(CUtensorMap* map, const void* x, const Prob& p, bool bf16) {
  const uint64_t dims[2] = {(uint64_t)p.C, (uint64_t)p.B * p.N};
  const uint64_t strides[1] = {(uint64_t)p.C * 2};
  const uint32_t box[2] = {64, 1};
  return encode_tiled_map(map, bf16, 2, x, dims, strides, box, "tc forward");
}

template <int D, bool BF16>
int tcf_forward_t(const ow_bigemm_args_t* a, const Prob& p, const unsigned char* img, const uint16_t* amat,
                  const float* gg, const float* nwc, const int* layout, cudaStream_t st) {
  CUtensorMap map;
  OW_RETURN_IF(make_xmap(&map, a->x, p, BF16));
  int* fault = nullptr;
  OW_RETURN_IF(fault_word(&fault));
  const int64_t items = (int64_t)p.Qc * ((p.BQ() + 7) / 8);
  const int grid = (int)std::min<int64_t>(items, device_sm_count());
  if (grid == 0) return OW_OK;
  const BlockArgs blk{(const float*)a->rstd, nwc, a->x};
  auto go = [&](auto* to, auto res) -> int {
    using TO = std::remove_pointer_t<decltype(to)>;
    auto kern = tcf_kernel<D, BF16, TO, decltype(res)::value>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, FC<D>::SMEM);
    if (e != cudaSuccess) {
      set_error("tc forward: cannot reserve %d bytes of shared memory: %s", FC<D>::SMEM, cudaGetErrorString(e));
      return OW_ERR_CUDA;
    }
    profile_mark(OW_PROF_FWD, false, st);
    launch(kern, grid, THREADS, FC<D>::SMEM, st, map, p, img, amat, gg, layout, a->sample_scale, (TO*)a->out,
           blk, fault, wait_probe_ns());
    profile_mark(OW_PROF_FWD, true, st);
    OW_CHECK_LAUNCH("tcf_kernel");
    return OW_OK;
  };
  using T16 = std::conditional_t<BF16, __nv_bfloat16, __half>;
  const bool o16 = a->out_dtype == (BF16 ? OW_DTYPE_BF16 : OW_DTYPE_F16);
  if (a->rstd) return o16 ? go((T16*)nullptr, std::true_type{}) : go((float*)nullptr, std::true_type{});
  return o16 ? go((T16*)nullptr, std::false_type{}) : go((float*)nullptr, std::false_type{});
}

}  // namespace

// cuTensorMapEncodeTiled, looked up through the runtime once (the library
// does not link the driver library, so it loads on machines without one).
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    else
      cudaGetLastError();
  });
  return fn;
}

int encode_tiled_map(void* map, bool bf16, int rank, const void* base, const uint64_t* dims,
                     const uint64_t* strides, const uint32_t* box, const char* who) {
  auto encode = encode_fn();
  if (!encode) {
    set_error("%s: cuTensorMapEncodeTiled is not available from the CUDA driver", who);
    return OW_ERR_CUDA;
  }
  if (rank < 1 || rank > 5) {
    set_error("%s: tensor map rank %d", who, rank);
    return OW_ERR_INVALID;
  }
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i + 1 < rank) s[i] = strides[i];
  }
  const CUresult r = encode(static_cast<CUtensorMap*>(map),
                            bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                            (cuuint32_t)rank, const_cast<void*>(base), d, s, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("%s: cuTensorMapEncodeTiled failed (CUresult %d)", who, (int)r);
    return OW_ERR_CUDA;
  }
  return OW_OK;
}

bool tcf_covers(const ow_bigemm_args_t* a, const Prob& p) {
  const int c16 = a->compute_dtype;
  // Operator mode, or block mode (rstd given and the residual added).
  return (c16 == OW_DTYPE_BF16 || c16 == OW_DTYPE_F16) && a->x_dtype == c16 && (!a->rstd) == (!a->residual) &&
         p.chs == 1 && (p.d == 64 || p.d == 128) && p.rd == 2 * p.d && p.C % 8 == 0 &&
         (uintptr_t)a->x % 16 == 0 && (uintptr_t)a->out % 16 == 0 &&
         (a->out_dtype == c16 || a->out_dtype == OW_DTYPE_F32) &&
         (int64_t)p.B * p.N < (1LL << 31) - 1;
}

int tcf_forward(const ow_bigemm_args_t* a, const Prob& p, const unsigned char* img, const uint16_t* amat,
                const float* gg, const float* nwc, const int* layout, void* stream) {
  cudaStream_t st = (cudaStream_t)stream;
  const bool bf = a->compute_dtype == OW_DTYPE_BF16;
  if (p.d == 64)
    return bf ? tcf_forward_t<64, true>(a, p, img, amat, gg, nwc, layout, st)
              : tcf_forward_t<64, false>(a, p, img, amat, gg, nwc, layout, st);
  return bf ? tcf_forward_t<128, true>(a, p, img, amat, gg, nwc, layout, st)
            : tcf_forward_t<128, false>(a, p, img, amat, gg, nwc, layout, st);
}

}  // namespace ow
