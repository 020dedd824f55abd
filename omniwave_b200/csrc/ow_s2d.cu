// Space-to-depth + Linear on the tensor cores (sm_100a): the OmniWeave-T stem
// and downsamples, ``Linear(space_to_depth(x, f))`` (reference
// omniweave/models/backbone.py:14-27, :121, :128-132, :173-187), as one GEMM
// whose A rows are read from x in place, so the rearranged tensor
// [B, H/f, W/f, f f C] is never written:
//
//   out[m, n] = sum_k s2d(x)[m, k] W[n, k],   m = (b, i, j),  k = (dy, dx, c)
//
// Two kernels share the pipeline (persistent grid, one CTA per SM, a 4-stage
// shared-memory ring for A and B, a double-buffered TMEM accumulator so the
// epilogue of one tile overlaps the main loop of the next):
//
// * downsample (x NHWC, 16-bit): one thread loads each A stage with a 5-D TMA
//   box over x viewed as [B Ho, f (dy), Wo, f (dx), C]; for a fixed k chunk
//   (dy, dx, 64 channels) the box {64 ch, 1, Wo, 1, R} holds rows m of R whole
//   output rows (R = floor(128 / Wo)), already in the 128-byte-swizzled
//   K-major layout the MMA reads.  Tiles have R Wo <= 128 rows, 256 features.
// * stem (x NCHW, f = 4, C = 3, K = 48): eight gather warps in two groups
//   fill alternate stages, one output row per thread from twelve 16-byte
//   loads (4 dx values of one (c, dy) each), rounding f32 to the compute
//   type as autocast does; the weight images stay resident.
//
// * depth-to-space (the input gradient of the downsample): the same
//   pipeline with A = the gradient rows y [B Ho Wo, N] (a 3-D TMA box of R
//   whole rows) and the weight read transposed, so the GEMM produces
//   s2d-ordered features k = (dy, dx, c); the epilogue stores every
//   32-feature chunk (one (dy, dx) block, 32 channels) at its place in the
//   NHWC image [B, f Ho, f Wo, C], in f32 or the compute type.
//
// Weights go through a prep kernel into pre-swizzled K-major images of the
// compute type (128 or 256 features x 64 K).  The epilogue converts the f32
// accumulator to the compute type and leaves through a per-warp staging
// buffer as whole 64-byte row segments.  Every wait is bounded (ow_sm100.cuh).

#include <cuda.h>

#include <algorithm>
#include <type_traits>

#include "ow_common.cuh"
#include "ow_internal.h"
#include "ow_sm100.cuh"

namespace ow {
namespace {

using namespace sm100;

constexpr int TM = 128;          // accumulator rows (TMEM lanes)
constexpr int KE = 64;           // K elements per stage (one 128-byte line of 16-bit values)
constexpr int A_ST = TM * 128;   // 16 KB
constexpr int STG_W = 2048;      // epilogue staging per warp: 32 rows x 32 features x 2 bytes

// Kernel-shape constants.  SN: features per tile; PRODW: warps that fill the
// A stages (one thread issues TMA for the downsample); the MMA warp and four
// epilogue warps follow them.  The downsample streams A and B through the
// ring (4 stages at SN = 256, 6 at SN = 128); the stem keeps its weight
// images resident and streams A alone.
template <bool STEM_, int SN_>
struct SC {
  static constexpr bool STEM = STEM_;
  static constexpr int SN = SN_;
  static constexpr int STAGES = (STEM || SN == 256) ? 4 : 6;
  static constexpr int B_ST = SN * 128;
  static constexpr int PRODW = STEM ? 8 : 1;
  static constexpr int MMA_W = PRODW;
  static constexpr int EPI_W = PRODW + 1;
  static constexpr int THREADS = (PRODW + 5) * 32;
  static constexpr int MAX_NT = STEM ? 4 : 0;          // stem: resident weight images
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = STAGES * A_ST;
  static constexpr int B_BYTES = STEM ? MAX_NT * B_ST : STAGES * B_ST;
  static constexpr int OFF_STG = OFF_B + B_BYTES;
  static constexpr int OFF_BAR = OFF_STG + 4 * STG_W;
  static constexpr int NBAR = 2 * STAGES + 4 + 2;      // full, empty, tfull[2], tfree[2], weights, probe
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;
  static constexpr int TMEM_COLS = 2 * SN;
  static_assert(SN == 128 || SN == 256, "feature tile");
  static_assert(SMEM <= 232448, "shared memory budget");
  static_assert(TMEM_COLS <= 512, "TMEM budget");
};
using StemK = SC<true, 128>;

struct S2dArgs {
  const void* x;
  int B, H, W, C, f;
  int Ho, Wo;
  int R, MT;             // downsample: output rows per tile (R) and tile rows R Wo; stem: MT = 128
  int64_t M;             // B Ho Wo
  int mtiles, NT, KC;    // row tiles, feature tiles, 64-wide K chunks
  int N;
  const unsigned char* wimg;  // [NT][KC] images of SN x 64 (SW128 K-major)
  void* out;
  int oC, oW;            // depth-to-space output: channels and width (f Wo) of the image
  int* fault;
  uint32_t probe_ns;
};

// 5-D TMA tile load into shared memory, completing on ``bar``.
__device__ __forceinline__ void tma_load_5d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            int c4, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(smem_u32(bar))
      : "memory");
}

// 3-D TMA tile load into shared memory, completing on ``bar``.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

// Weight images: W[n, k] -> image (n / SN, k / 64), row n % SN, column
// k % 64, SW128 K-major, in the compute type; columns k >= K are zero.
// TR: the weight is stored transposed, W[n, k] at w[k N + n].
template <typename TW, typename T16, int SN, bool TR = false>
__global__ void s2d_wprep_kernel(const TW* __restrict__ w, int N, int K, int KC, unsigned char* __restrict__ img) {
  const int64_t total = (int64_t)N * KC * KE;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int n = (int)(i / (KC * KE)), k = (int)(i - (int64_t)n * KC * KE);
    const float v = k < K ? load_as<float>(w, TR ? (int64_t)k * N + n : (int64_t)n * K + k) : 0.f;
    unsigned char* base = img + ((int64_t)(n / SN) * KC + k / KE) * (SN * 128);
    *reinterpret_cast<T16*>(base + sw128_off(n % SN, k % KE, SN)) = Elem<T16>::from(v);
  }
}

// Output modes of the epilogue: OUT_ROWS writes tile row m as out row m (the
// compute type); OUT_D2S16 / OUT_D2S32 write feature k = (dy, dx, c) of row
// m = (b, i, j) to pixel (b, f i + dy, f j + dx), channel c of an NHWC image
// with oC channels and width oW (depth-to-space), in the compute type or as
// f32 holding the compute-type rounding (what the reference's autocast
// backward produces: a 16-bit GEMM output cast to the f32 input's dtype).
constexpr int OUT_ROWS = 0, OUT_D2S16 = 1, OUT_D2S32 = 2;

// Epilogue of one tile for the calling warp.  A warp may only read the TMEM
// lane quarter q = (warp id) % 4, which holds tile rows 32 q .. 32 q + 31.
// Per 32-feature chunk the warp converts its 32 x 32 block, stages it in
// ``stg`` (16-byte units rotated by the row pair, conflict free both ways)
// and stores 8 rows x 64 bytes per instruction (f32: the chunk in two
// 16-feature halves).
template <int SN, bool BF16, int OM>
__device__ __forceinline__ void epilogue_tile(uint32_t tacc, unsigned char* stg, const S2dArgs& a, int64_t mrow0,
                                              int ncol0) {
  using T16 = std::conditional_t<BF16, __nv_bfloat16, __half>;
  const int lane = threadIdx.x & 31, q = (threadIdx.x >> 5) & 3;
  // Element offset of the start of each row this lane stores (it = 0..3),
  // -1 for rows past the tile or the matrix.  Depth-to-space: tile row r is
  // output row (mrow0 / Wo + r / Wo, r % Wo) of y, i.e. pixel
  // (f (mrow0 / Wo + r / Wo), f (r % Wo)) before the (dy, dx) of the chunk.
  int64_t rowoff[4];
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int r = q * 32 + it * 8 + (lane >> 2);
    const int64_t m = mrow0 + r;
    if (r >= a.MT || m >= a.M) {
      rowoff[it] = -1;
    } else if constexpr (OM == OUT_ROWS) {
      rowoff[it] = m * a.N;
    } else {
      const int io = r / a.Wo, j = r - io * a.Wo;
      const int64_t bi = mrow0 / a.Wo + io;
      rowoff[it] = (bi * a.f * a.oW + (int64_t)a.f * j) * a.oC;
    }
  }
#pragma unroll 1
  for (int cb = 0; cb < SN / 32; ++cb) {
    uint32_t v[32];
    tmem_ld32(tacc + ((uint32_t)(q * 32) << 16) + cb * 32, v);
    tmem_ld_wait();
    // Offset of the chunk's first feature inside a row (depth-to-space: the
    // chunk is 32 channels of one (dy, dx) block).
    int64_t coff = ncol0 + cb * 32;
    if constexpr (OM != OUT_ROWS) {
      const int k0 = ncol0 + cb * 32, blk = k0 / a.oC, c0 = k0 - blk * a.oC;
      const int dy = blk / a.f, dx = blk - dy * a.f;
      coff = ((int64_t)dy * a.oW + dx) * a.oC + c0;
    }
    if constexpr (OM == OUT_D2S32) {
      float* out = reinterpret_cast<float*>(a.out);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          auto rd = [&](int i) {
            return __float_as_uint(Elem<T16>::to_f(Elem<T16>::from(__uint_as_float(v[16 * h + 4 * u + i]))));
          };
          const uint4 o = make_uint4(rd(0), rd(1), rd(2), rd(3));
          *reinterpret_cast<uint4*>(stg + lane * 64 + ((u ^ ((lane >> 1) & 3)) << 4)) = o;
        }
        __syncwarp();
#pragma unroll
        for (int it = 0; it < 4; ++it) {
          const int row = it * 8 + (lane >> 2), pc = lane & 3;
          const uint4 o = *reinterpret_cast<const uint4*>(stg + row * 64 + ((pc ^ ((row >> 1) & 3)) << 4));
          if (rowoff[it] >= 0) *reinterpret_cast<uint4*>(out + rowoff[it] + coff + 16 * h + pc * 4) = o;
        }
        __syncwarp();
      }
    } else {
      T16* out = reinterpret_cast<T16*>(a.out);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        uint4 o;
        o.x = pack2<BF16>(__uint_as_float(v[8 * u + 0]), __uint_as_float(v[8 * u + 1]));
        o.y = pack2<BF16>(__uint_as_float(v[8 * u + 2]), __uint_as_float(v[8 * u + 3]));
        o.z = pack2<BF16>(__uint_as_float(v[8 * u + 4]), __uint_as_float(v[8 * u + 5]));
        o.w = pack2<BF16>(__uint_as_float(v[8 * u + 6]), __uint_as_float(v[8 * u + 7]));
        *reinterpret_cast<uint4*>(stg + lane * 64 + ((u ^ ((lane >> 1) & 3)) << 4)) = o;
      }
      __syncwarp();
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        const int row = it * 8 + (lane >> 2), pc = lane & 3;
        const uint4 o = *reinterpret_cast<const uint4*>(stg + row * 64 + ((pc ^ ((row >> 1) & 3)) << 4));
        if (rowoff[it] >= 0) *reinterpret_cast<uint4*>(out + rowoff[it] + coff + pc * 8) = o;
      }
      __syncwarp();
    }
  }
}

// One thread: the MMAs of every tile this CTA owns.  Ring stage g (g counts
// K chunks over all tiles) holds A at OFF_A and B at OFF_B (the stem reads
// the resident weight image of the tile's feature block instead).
template <class K, bool BF16>
__device__ __forceinline__ void mma_loop(unsigned char* sm, uint64_t* full, uint64_t* empty, uint64_t* tfull,
                                         uint64_t* tfree, uint64_t* bar_w, uint32_t tbase, const S2dArgs& a,
                                         int ntiles, volatile int* abort) {
  constexpr bool STEM = K::STEM;
  constexpr int STAGES = K::STAGES;
  constexpr uint32_t ID = idesc_f16(TM, K::SN, BF16);
  constexpr int KSTEPS = STEM ? 3 : KE / 16;   // the stem's K is 48
  const uint32_t s0 = smem_u32(sm);
  if (STEM && !mbar_wait(bar_w, 0, abort)) return;
  int g = 0, tl = 0;
  for (int t = blockIdx.x; t < ntiles && !*abort; t += gridDim.x, ++tl) {
    const int acc = tl & 1;
    if (tl >= 2 && !mbar_wait(tfree + acc, ((tl >> 1) - 1) & 1, abort)) break;
    tc_fence_after();
    const int nt = t % a.NT;
    const uint32_t tacc = tbase + acc * K::SN;
    for (int kc = 0; kc < a.KC; ++kc, ++g) {
      const int s = g % STAGES;
      if (!mbar_wait(full + s, (g / STAGES) & 1, abort)) break;
      tc_fence_after();
      const uint32_t aA = s0 + K::OFF_A + s * A_ST;
      const uint32_t aB = s0 + K::OFF_B + (STEM ? nt * K::B_ST : s * K::B_ST);
#pragma unroll
      for (int kk = 0; kk < KSTEPS; ++kk)
        umma_f16(tacc, sdesc_sw128(sw128_kstep(aA, kk, TM)), sdesc_sw128(sw128_kstep(aB, kk, K::SN)), ID,
                 (kc > 0 || kk > 0) ? 1u : 0u);
      umma_commit(empty + s);
    }
    umma_commit(tfull + acc);
  }
}

template <class K, bool BF16, int OM = OUT_ROWS>
__device__ __forceinline__ void epilogue_loop(unsigned char* sm, uint64_t* tfull, uint64_t* tfree, uint32_t tbase,
                                              const S2dArgs& a, int ntiles, volatile int* abort) {
  const int w = (threadIdx.x >> 5) - K::EPI_W;
  unsigned char* stg = sm + K::OFF_STG + w * STG_W;
  int tl = 0;
  for (int t = blockIdx.x; t < ntiles && !*abort; t += gridDim.x, ++tl) {
    const int acc = tl & 1;
    if (!mbar_wait(tfull + acc, (tl >> 1) & 1, abort)) break;
    __syncwarp();
    tc_fence_after();
    const int mt = t / a.NT, nt = t % a.NT;
    epilogue_tile<K::SN, BF16, OM>(tbase + acc * K::SN, stg, a, (int64_t)mt * a.MT, nt * K::SN);
    tc_fence_before();
    mbar_arrive(tfree + acc);
  }
}

// Barrier block shared by both kernels.
struct Bars {
  uint64_t *full, *empty, *tfull, *tfree, *w, *probe;
  uint32_t* tmem;
  volatile int* abort;
};

template <class K>
__device__ __forceinline__ Bars carve_bars(unsigned char* sm) {
  uint64_t* b = reinterpret_cast<uint64_t*>(sm + K::OFF_BAR);
  Bars r;
  r.full = b;
  r.empty = b + K::STAGES;
  r.tfull = b + 2 * K::STAGES;
  r.tfree = r.tfull + 2;
  r.w = r.tfree + 2;
  r.probe = r.w + 1;
  r.tmem = reinterpret_cast<uint32_t*>(b + K::NBAR);
  r.abort = reinterpret_cast<volatile int*>(r.tmem + 1);
  return r;
}

// Thread 0 initialises the barriers (``full`` takes ``full_count`` arrivals)
// and runs the wait-timeout self-check; the MMA warp allocates TMEM.
template <class K>
__device__ __forceinline__ uint32_t setup(const Bars& B, int full_count, uint32_t probe_ns) {
  if (threadIdx.x == 0) {
    for (int s = 0; s < K::STAGES; ++s) {
      mbar_init(B.full + s, full_count);
      mbar_init(B.empty + s, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(B.tfull + i, 1);
      mbar_init(B.tfree + i, 128);
    }
    mbar_init(B.w, 1);
    mbar_init(B.probe, 1);
    *B.abort = 0;
    fence_mbar_init();
    wait_probe(B.probe, B.abort, probe_ns);
  }
  if ((int)(threadIdx.x >> 5) == K::MMA_W) tmem_alloc(B.tmem, K::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  return *B.tmem;
}

template <class K>
__device__ __forceinline__ void teardown(const Bars& B, uint32_t tbase, int* fault) {
  __syncwarp();
  __syncthreads();
  report_abort(B.abort, fault);
  if (*B.abort) {
    // A wait gave up: give in-flight copies and MMAs time to land before
    // the shared memory and TMEM they target are released.
    for (int i = 0; i < 1000; ++i) __nanosleep(1000);
  }
  if ((int)(threadIdx.x >> 5) == K::MMA_W) {
    tc_fence_after();
    tmem_dealloc(tbase, K::TMEM_COLS);
  }
}

// ---------------------------------------------------------------- downsample
// OM == OUT_ROWS: the downsample, A rows through the 5-D box over x.
// Depth-to-space modes: A = the gradient rows y through a 3-D box
// {64, Wo, R} over y viewed as [B Ho, Wo, K] (the same R whole rows).
template <int SN, bool BF16, int OM = OUT_ROWS>
__global__ void __launch_bounds__(SC<false, SN>::THREADS, 1)
    s2d_ds_kernel(const __grid_constant__ CUtensorMap xmap, S2dArgs a) {
  using K = SC<false, SN>;
  constexpr int STAGES = K::STAGES;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const Bars B = carve_bars<K>(sm);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntiles = a.mtiles * a.NT;
  const uint32_t tbase = setup<K>(B, 1, a.probe_ns);

  if (*B.abort) {
    // the wait-timeout self-check ran out: nothing is issued
  } else if (warp == 0) {
    if (lane == 0) {
      const uint32_t bytes = (uint32_t)(a.MT * 128 + K::B_ST);
      int g = 0;
      for (int t = blockIdx.x; t < ntiles && !*B.abort; t += gridDim.x) {
        const int mt = t / a.NT, nt = t % a.NT;
        for (int kc = 0; kc < a.KC; ++kc, ++g) {
          const int s = g % STAGES;
          if (g >= STAGES && !mbar_wait(B.empty + s, ((g / STAGES) - 1) & 1, B.abort)) break;
          const int k0 = kc * KE;
          mbar_arrive_expect_tx(B.full + s, bytes);
          if constexpr (OM == OUT_ROWS) {
            const int dy = k0 / (a.f * a.C), dx = (k0 / a.C) % a.f, c0 = k0 % a.C;
            tma_load_5d(sm + K::OFF_A + s * A_ST, &xmap, c0, dx, 0, dy, mt * a.R, B.full + s);
          } else {
            tma_load_3d(sm + K::OFF_A + s * A_ST, &xmap, k0, 0, mt * a.R, B.full + s);
          }
          bulk_g2s(sm + K::OFF_B + s * K::B_ST, a.wimg + ((int64_t)nt * a.KC + kc) * K::B_ST, K::B_ST, B.full + s);
        }
      }
    }
  } else if (warp == K::MMA_W) {
    if (lane == 0) mma_loop<K, BF16>(sm, B.full, B.empty, B.tfull, B.tfree, B.w, tbase, a, ntiles, B.abort);
  } else {
    epilogue_loop<K, BF16, OM>(sm, B.tfull, B.tfree, tbase, a, ntiles, B.abort);
  }
  teardown<K>(B, tbase, a.fault);
}

// ---------------------------------------------------------------- stem
template <typename TX, bool BF16>
__global__ void __launch_bounds__(StemK::THREADS, 1) s2d_stem_kernel(S2dArgs a) {
  using K = StemK;
  constexpr int STAGES = K::STAGES;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const Bars B = carve_bars<K>(sm);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntiles = a.mtiles * a.NT;
  const uint32_t tbase = setup<K>(B, 128, a.probe_ns);

  if (*B.abort) {
    // the wait-timeout self-check ran out: nothing is issued
  } else if (warp < K::PRODW) {
    // Gather group gp fills the stages of this CTA's tiles lt = gp, gp + 2, ...
    const int gp = warp >> 2, r = threadIdx.x & 127;
    const TX* x = reinterpret_cast<const TX*>(a.x);
    const int64_t hw = (int64_t)a.Ho * a.Wo;
    int lt = gp;
    for (int t = blockIdx.x + gp * gridDim.x; t < ntiles && !*B.abort; t += 2 * gridDim.x, lt += 2) {
      const int s = lt % STAGES;
      if (lt >= STAGES && !mbar_wait(B.empty + s, ((lt / STAGES) - 1) & 1, B.abort)) break;
      const int64_t m = (int64_t)(t / a.NT) * TM + r;
      float v[3][4][4];  // [c][dy][dx]
      if (m < a.M) {
        const int b = (int)(m / hw);
        const int rem = (int)(m - (int64_t)b * hw);
        const int i = rem / a.Wo, j = rem - i * a.Wo;
#pragma unroll
        for (int c = 0; c < 3; ++c)
#pragma unroll
          for (int dy = 0; dy < 4; ++dy) {
            const int64_t off = (((int64_t)b * 3 + c) * a.H + 4 * i + dy) * a.W + 4 * j;
            if constexpr (sizeof(TX) == 4) {
              const float4 f4 = __ldg(reinterpret_cast<const float4*>(x + off));
              v[c][dy][0] = f4.x; v[c][dy][1] = f4.y; v[c][dy][2] = f4.z; v[c][dy][3] = f4.w;
            } else {
              const uint2 h = __ldg(reinterpret_cast<const uint2*>(x + off));
              const float2 lo = unpack2<BF16>(h.x), hi = unpack2<BF16>(h.y);
              v[c][dy][0] = lo.x; v[c][dy][1] = lo.y; v[c][dy][2] = hi.x; v[c][dy][3] = hi.y;
            }
          }
      } else {
#pragma unroll
        for (int c = 0; c < 3; ++c)
#pragma unroll
          for (int dy = 0; dy < 4; ++dy)
#pragma unroll
            for (int dx = 0; dx < 4; ++dx) v[c][dy][dx] = 0.f;
      }
      // k = 12 dy + 3 dx + c; 16-byte chunk ch of the row holds k = 8 ch .. 8 ch + 7
      unsigned char* st = sm + K::OFF_A + s * A_ST + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
      for (int ch = 0; ch < 6; ++ch) {
        uint32_t pk[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int k0 = 8 * ch + 2 * e, k1 = k0 + 1;
          pk[e] = pack2<BF16>(v[k0 % 3][k0 / 12][(k0 % 12) / 3], v[k1 % 3][k1 / 12][(k1 % 12) / 3]);
        }
        *reinterpret_cast<uint4*>(st + ((ch ^ (r & 7)) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
      fence_proxy_async_smem();
      mbar_arrive(B.full + s);
    }
  } else if (warp == K::MMA_W) {
    if (lane == 0) {
      mbar_arrive_expect_tx(B.w, (uint32_t)(a.NT * K::B_ST));
      for (int nt = 0; nt < a.NT; ++nt)
        bulk_g2s(sm + K::OFF_B + nt * K::B_ST, a.wimg + (int64_t)nt * K::B_ST, K::B_ST, B.w);
      mma_loop<K, BF16>(sm, B.full, B.empty, B.tfull, B.tfree, B.w, tbase, a, ntiles, B.abort);
    }
  } else {
    epilogue_loop<K, BF16>(sm, B.tfull, B.tfree, tbase, a, ntiles, B.abort);
  }
  teardown<K>(B, tbase, a.fault);
}

bool is16(int dt) { return dt == OW_DTYPE_BF16 || dt == OW_DTYPE_F16; }

int s2d_check(const ow_s2d_linear_t* a, const char** why) {
  auto no = [&](const char* m) {
    if (why) *why = m;
    return OW_ERR_UNSUPPORTED;
  };
  if (!a) return no("args is NULL");
  if (a->batch <= 0 || a->height <= 0 || a->width <= 0 || a->channels <= 0 || a->factor <= 0)
    return no("batch, height, width, channels and factor must be positive");
  if (a->height % a->factor || a->width % a->factor) return no("height and width must be divisible by factor");
  if (!is16(a->out_dtype)) return no("out dtype must be bfloat16 or float16");
  if (a->w_dtype != OW_DTYPE_F32 && a->w_dtype != a->out_dtype)
    return no("weight dtype must be float32 or the out dtype");
  if ((int64_t)a->batch * a->height * a->width * a->channels >= (1LL << 40)) return no("x too large");
  if ((int64_t)a->batch * (a->height / a->factor) * (a->width / a->factor) >= (1LL << 31) - TM)
    return no("too many output rows");
  if (a->layout == OW_LAYOUT_NHWC) {
    if (a->x_dtype != a->out_dtype) return no("NHWC: x dtype must equal the out dtype");
    if (a->channels % KE) return no("NHWC: channels must be a multiple of 64");
    if (a->width / a->factor > TM) return no("NHWC: width / factor must be at most 128");
    if (a->out_features <= 0 || a->out_features % 256)
      return no("NHWC: out_features must be a multiple of 256");
  } else if (a->layout == OW_LAYOUT_NCHW) {
    if (a->channels != 3 || a->factor != 4) return no("NCHW: only channels == 3 and factor == 4 (the stem)");
    if (a->x_dtype != OW_DTYPE_F32 && a->x_dtype != a->out_dtype)
      return no("NCHW: x dtype must be float32 or the out dtype");
    if (a->out_features <= 0 || a->out_features % StemK::SN || a->out_features > StemK::MAX_NT * StemK::SN)
      return no("NCHW: out_features must be a multiple of 128, at most 512");
  } else {
    return no("layout must be OW_LAYOUT_NHWC or OW_LAYOUT_NCHW");
  }
  return OW_OK;
}

size_t wimg_bytes(const ow_s2d_linear_t* a) {
  const int K = a->factor * a->factor * a->channels;
  const int KC = (K + KE - 1) / KE;
  return (size_t)a->out_features * KC * KE * 2;
}

int d2s_check(const ow_d2s_linear_t* a, const char** why) {
  auto no = [&](const char* m) {
    if (why) *why = m;
    return OW_ERR_UNSUPPORTED;
  };
  if (!a) return no("args is NULL");
  if (a->batch <= 0 || a->height <= 0 || a->width <= 0 || a->channels <= 0 || a->factor <= 0 ||
      a->in_features <= 0)
    return no("batch, height, width, channels, factor and in_features must be positive");
  if (a->height % a->factor || a->width % a->factor) return no("height and width must be divisible by factor");
  if (!is16(a->y_dtype)) return no("y dtype must be bfloat16 or float16");
  if (a->w_dtype != OW_DTYPE_F32 && a->w_dtype != a->y_dtype) return no("weight dtype must be float32 or y's dtype");
  if (a->out_dtype != OW_DTYPE_F32 && a->out_dtype != a->y_dtype) return no("out dtype must be float32 or y's dtype");
  if (a->channels % KE) return no("channels must be a multiple of 64");
  if (a->in_features % KE) return no("in_features must be a multiple of 64");
  if ((int64_t)a->factor * a->factor * a->channels % 256) return no("factor^2 * channels must be a multiple of 256");
  if (a->width / a->factor > TM) return no("width / factor must be at most 128");
  if ((int64_t)a->batch * a->height * a->width * a->channels >= (1LL << 40)) return no("out too large");
  if ((int64_t)a->batch * (a->height / a->factor) * (a->width / a->factor) >= (1LL << 31) - TM)
    return no("too many rows");
  return OW_OK;
}

}  // namespace
}  // namespace ow

using namespace ow;

extern "C" {

size_t ow_s2d_linear_workspace_size(const ow_s2d_linear_t* a) {
  if (s2d_check(a, nullptr) != OW_OK) return 0;
  return wimg_bytes(a) + 256;
}

int ow_s2d_linear_fwd(const ow_s2d_linear_t* a, void* stream) {
  clear_error();
  const char* why = nullptr;
  if (s2d_check(a, &why) != OW_OK) {
    set_error("ow_s2d_linear_fwd: %s", why);
    return OW_ERR_UNSUPPORTED;
  }
  OW_CHECK_ARG(a->x && a->weight && a->out, "ow_s2d_linear_fwd: a pointer is NULL");
  OW_CHECK_ARG((uintptr_t)a->x % 16 == 0 && (uintptr_t)a->out % 16 == 0,
               "ow_s2d_linear_fwd: x and out must be 16-byte aligned");
  const size_t need = ow_s2d_linear_workspace_size(a);
  if (!a->workspace || a->workspace_bytes < need) {
    set_error("ow_s2d_linear_fwd needs %zu workspace bytes, got %zu", need, a->workspace_bytes);
    return OW_ERR_WORKSPACE;
  }
  cudaStream_t st = (cudaStream_t)stream;
  const bool stem = a->layout == OW_LAYOUT_NCHW;
  const bool bf = a->out_dtype == OW_DTYPE_BF16;
  S2dArgs k{};
  k.x = a->x;
  k.B = a->batch; k.H = a->height; k.W = a->width; k.C = a->channels; k.f = a->factor;
  k.Ho = a->height / a->factor; k.Wo = a->width / a->factor;
  k.M = (int64_t)k.B * k.Ho * k.Wo;
  k.N = a->out_features;
  const int K = k.f * k.f * k.C;
  k.KC = (K + KE - 1) / KE;
  const int sms = device_sm_count();
  int sn = StemK::SN;
  if (stem) {
    k.R = 0;
    k.MT = TM;
    k.mtiles = (int)((k.M + TM - 1) / TM);
  } else {
    k.R = TM / k.Wo;
    k.MT = k.R * k.Wo;
    k.mtiles = (int)(((int64_t)k.B * k.Ho + k.R - 1) / k.R);
    // Feature tiles of 256 (twice the reuse of each A stage) unless 128
    // fills the waves of the persistent grid far better.
    auto fill = [&](int w) {
      const int64_t t = (int64_t)k.mtiles * (k.N / w);
      return (double)t / (double)(((t + sms - 1) / sms) * sms);
    };
    sn = fill(128) > fill(256) + 0.25 ? 128 : 256;
  }
  k.NT = k.N / sn;
  unsigned char* img = (unsigned char*)(((uintptr_t)a->workspace + 255) & ~(uintptr_t)255);
  k.wimg = img;
  k.out = a->out;
  OW_RETURN_IF(fault_word(&k.fault));
  k.probe_ns = wait_probe_ns();

  {  // weight images
    const int64_t nw = (int64_t)k.N * k.KC * KE;
    const int pg = (int)std::min<int64_t>((nw + 255) / 256, (int64_t)sms * 8);
    auto prep = [&](auto* tw, auto* t16) {
      using TW = std::remove_pointer_t<decltype(tw)>;
      using T16 = std::remove_pointer_t<decltype(t16)>;
      if (sn == 128)
        launch(s2d_wprep_kernel<TW, T16, 128>, pg, 256, 0, st, (const TW*)a->weight, k.N, K, k.KC, img);
      else
        launch(s2d_wprep_kernel<TW, T16, 256>, pg, 256, 0, st, (const TW*)a->weight, k.N, K, k.KC, img);
    };
    if (bf) {
      if (a->w_dtype == OW_DTYPE_F32) prep((float*)nullptr, (__nv_bfloat16*)nullptr);
      else prep((__nv_bfloat16*)nullptr, (__nv_bfloat16*)nullptr);
    } else {
      if (a->w_dtype == OW_DTYPE_F32) prep((float*)nullptr, (__half*)nullptr);
      else prep((__half*)nullptr, (__half*)nullptr);
    }
    OW_CHECK_LAUNCH("s2d_wprep_kernel");
  }

  const int ntiles = k.mtiles * k.NT;
  const int grid = std::min(ntiles, sms);
  if (grid <= 0) return OW_OK;
  auto attr = [&](const void* kern, int smem) -> int {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) {
      set_error("s2d linear: cannot reserve %d bytes of shared memory: %s", smem, cudaGetErrorString(e));
      return OW_ERR_CUDA;
    }
    return OW_OK;
  };
  if (stem) {
    auto go = [&](auto kern) -> int {
      OW_RETURN_IF(attr((const void*)kern, StemK::SMEM));
      launch(kern, grid, StemK::THREADS, StemK::SMEM, st, k);
      OW_CHECK_LAUNCH("s2d_stem_kernel");
      return OW_OK;
    };
    if (a->x_dtype == OW_DTYPE_F32)
      return bf ? go(s2d_stem_kernel<float, true>) : go(s2d_stem_kernel<float, false>);
    return bf ? go(s2d_stem_kernel<__nv_bfloat16, true>) : go(s2d_stem_kernel<__half, false>);
  }

  // x viewed as [B Ho, f (dy), Wo, f (dx), C], listed innermost first
  CUtensorMap map;
  const uint64_t C = (uint64_t)k.C, f = (uint64_t)k.f, W = (uint64_t)k.W;
  const uint64_t dims[5] = {C, f, (uint64_t)k.Wo, f, (uint64_t)k.B * k.Ho};
  const uint64_t strides[4] = {C * 2, f * C * 2, W * C * 2, f * W * C * 2};
  const uint32_t box[5] = {(uint32_t)KE, 1, (uint32_t)k.Wo, 1, (uint32_t)k.R};
  OW_RETURN_IF(encode_tiled_map(&map, bf, 5, a->x, dims, strides, box, "s2d linear"));
  auto go = [&](auto kern, int smem, int threads) -> int {
    OW_RETURN_IF(attr((const void*)kern, smem));
    launch(kern, grid, threads, smem, st, map, k);
    OW_CHECK_LAUNCH("s2d_ds_kernel");
    return OW_OK;
  };
  using K128 = SC<false, 128>;
  using K256 = SC<false, 256>;
  if (sn == 128)
    return bf ? go(s2d_ds_kernel<128, true>, K128::SMEM, K128::THREADS)
              : go(s2d_ds_kernel<128, false>, K128::SMEM, K128::THREADS);
  return bf ? go(s2d_ds_kernel<256, true>, K256::SMEM, K256::THREADS)
            : go(s2d_ds_kernel<256, false>, K256::SMEM, K256::THREADS);
}

size_t ow_d2s_linear_workspace_size(const ow_d2s_linear_t* a) {
  if (d2s_check(a, nullptr) != OW_OK) return 0;
  const size_t nf = (size_t)a->factor * a->factor * a->channels;
  return nf * (size_t)a->in_features * 2 + 256;
}

int ow_d2s_linear_fwd(const ow_d2s_linear_t* a, void* stream) {
  clear_error();
  const char* why = nullptr;
  if (d2s_check(a, &why) != OW_OK) {
    set_error("ow_d2s_linear_fwd: %s", why);
    return OW_ERR_UNSUPPORTED;
  }
  OW_CHECK_ARG(a->y && a->weight && a->out, "ow_d2s_linear_fwd: a pointer is NULL");
  OW_CHECK_ARG((uintptr_t)a->y % 16 == 0 && (uintptr_t)a->out % 16 == 0,
               "ow_d2s_linear_fwd: y and out must be 16-byte aligned");
  const size_t need = ow_d2s_linear_workspace_size(a);
  if (!a->workspace || a->workspace_bytes < need) {
    set_error("ow_d2s_linear_fwd needs %zu workspace bytes, got %zu", need, a->workspace_bytes);
    return OW_ERR_WORKSPACE;
  }
  cudaStream_t st = (cudaStream_t)stream;
  const bool bf = a->y_dtype == OW_DTYPE_BF16;
  const int f = a->factor;
  S2dArgs k{};
  k.x = a->y;
  k.B = a->batch;
  k.H = a->height;
  k.W = a->width;
  k.f = f;
  k.C = a->in_features;
  k.Ho = a->height / f;
  k.Wo = a->width / f;
  k.M = (int64_t)k.B * k.Ho * k.Wo;
  k.N = f * f * a->channels;               // s2d-ordered features (dy, dx, c)
  k.KC = a->in_features / KE;
  k.R = TM / k.Wo;
  k.MT = k.R * k.Wo;
  k.mtiles = (int)(((int64_t)k.B * k.Ho + k.R - 1) / k.R);
  k.oC = a->channels;
  k.oW = a->width;
  const int sms = device_sm_count();
  auto fill = [&](int w) {
    const int64_t t = (int64_t)k.mtiles * (k.N / w);
    return (double)t / (double)(((t + sms - 1) / sms) * sms);
  };
  const int sn = fill(128) > fill(256) + 0.25 ? 128 : 256;
  k.NT = k.N / sn;
  unsigned char* img = (unsigned char*)(((uintptr_t)a->workspace + 255) & ~(uintptr_t)255);
  k.wimg = img;
  k.out = a->out;
  OW_RETURN_IF(fault_word(&k.fault));
  k.probe_ns = wait_probe_ns();

  {  // weight images of W^T: feature k' = (dy, dx, c), K = the input feature n
    const int64_t nw = (int64_t)k.N * k.KC * KE;
    const int pg = (int)std::min<int64_t>((nw + 255) / 256, (int64_t)sms * 8);
    auto prep = [&](auto* tw, auto* t16) {
      using TW = std::remove_pointer_t<decltype(tw)>;
      using T16 = std::remove_pointer_t<decltype(t16)>;
      if (sn == 128)
        launch(s2d_wprep_kernel<TW, T16, 128, true>, pg, 256, 0, st, (const TW*)a->weight, k.N, a->in_features,
               k.KC, img);
      else
        launch(s2d_wprep_kernel<TW, T16, 256, true>, pg, 256, 0, st, (const TW*)a->weight, k.N, a->in_features,
               k.KC, img);
    };
    if (bf) {
      if (a->w_dtype == OW_DTYPE_F32) prep((float*)nullptr, (__nv_bfloat16*)nullptr);
      else prep((__nv_bfloat16*)nullptr, (__nv_bfloat16*)nullptr);
    } else {
      if (a->w_dtype == OW_DTYPE_F32) prep((float*)nullptr, (__half*)nullptr);
      else prep((__half*)nullptr, (__half*)nullptr);
    }
    OW_CHECK_LAUNCH("s2d_wprep_kernel");
  }
  const int ntiles = k.mtiles * k.NT;
  const int grid = std::min(ntiles, sms);
  if (grid <= 0) return OW_OK;

  // y viewed as [B Ho, Wo, K], listed innermost first
  CUtensorMap map;
  const uint64_t K = (uint64_t)a->in_features;
  const uint64_t dims[3] = {K, (uint64_t)k.Wo, (uint64_t)k.B * k.Ho};
  const uint64_t strides[2] = {K * 2, (uint64_t)k.Wo * K * 2};
  const uint32_t box[3] = {(uint32_t)KE, (uint32_t)k.Wo, (uint32_t)k.R};
  OW_RETURN_IF(encode_tiled_map(&map, bf, 3, a->y, dims, strides, box, "d2s linear"));
  auto go = [&](auto kern, int smem, int threads) -> int {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) {
      set_error("d2s linear: cannot reserve %d bytes of shared memory: %s", smem, cudaGetErrorString(e));
      return OW_ERR_CUDA;
    }
    launch(kern, grid, threads, smem, st, map, k);
    OW_CHECK_LAUNCH("s2d_ds_kernel (depth-to-space)");
    return OW_OK;
  };
  using K128 = SC<false, 128>;
  using K256 = SC<false, 256>;
  const bool o32 = a->out_dtype == OW_DTYPE_F32;
  if (sn == 128) {
    if (bf) return o32 ? go(s2d_ds_kernel<128, true, OUT_D2S32>, K128::SMEM, K128::THREADS)
                       : go(s2d_ds_kernel<128, true, OUT_D2S16>, K128::SMEM, K128::THREADS);
    return o32 ? go(s2d_ds_kernel<128, false, OUT_D2S32>, K128::SMEM, K128::THREADS)
               : go(s2d_ds_kernel<128, false, OUT_D2S16>, K128::SMEM, K128::THREADS);
  }
  if (bf) return o32 ? go(s2d_ds_kernel<256, true, OUT_D2S32>, K256::SMEM, K256::THREADS)
                     : go(s2d_ds_kernel<256, true, OUT_D2S16>, K256::SMEM, K256::THREADS);
  return o32 ? go(s2d_ds_kernel<256, false, OUT_D2S32>, K256::SMEM, K256::THREADS)
             : go(s2d_ds_kernel<256, false, OUT_D2S16>, K256::SMEM, K256::THREADS);
}

}  // extern "C"
