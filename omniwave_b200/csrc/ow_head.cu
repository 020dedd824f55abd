// Global average pool + classifier head on the tensor cores (sm_100a), the
// tail of the OmniWeave backbone (reference omniweave/models/backbone.py:190-197,
// ``head(stage4.mean(dim=(1, 2)))``), as one kernel:
//
//   pooled[b, c] = round(inv_hw * sum_t x[b, t, c])          (compute type)
//   out[b, n]    = round(bias[n] + sum_c W[n, c] pooled[b, c])
//
// The pooled matrix never goes through global memory on the way to the head
// GEMM (it is written out only when the caller asks for it, for the
// backward).  A thread-block cluster of CL = 8 CTAs owns NB images (up to 32)
// and splits the channels eight ways: each CTA streams its channel slice of
// the NB feature maps from HBM, sums the tokens in f32, and writes the
// rounded means as the B operand of a tcgen05 MMA (SW128 K-major, one 64-
// channel chunk at a time) while TMA brings the matching 64-channel slice of
// every 128-class weight tile.  The MMA computes D[class, image] into TMEM
// (one 128 x MN f32 tile per 128 classes, MN = 16 or 32 image slots).  The
// eight partial logit blocks are then summed across the cluster through
// distributed shared memory: CTA r reads classes [128 r, 128 r + 128) of every
// peer in rank order, so the sum order is fixed and results are bitwise
// reproducible, and adds the bias (rounded to the compute type first, as
// autocast casts it; prefetched into shared memory at the start).
//
// The pool is HBM-bound, so the grid is one wave: the host asks the runtime
// how many 8-CTA clusters fit on the device at once and spreads the batch
// over that many clusters.  Every mbarrier wait is bounded (ow_sm100.cuh);
// the two cluster barriers are hardware barriers that every thread of every
// CTA reaches on every path.

#include <cuda.h>

#include <algorithm>
#include <mutex>
#include <type_traits>

#include "ow_common.cuh"
#include "ow_internal.h"
#include "ow_sm100.cuh"

namespace ow {
namespace {

using namespace sm100;

constexpr int CL = 8;                       // CTAs per cluster (channel split)
constexpr int TN = 128;                     // classes per MMA tile (M)
constexpr int MAX_NT = 8;                   // class tiles: classes <= 1024
constexpr int MAX_KCH = 4;                  // 64-channel chunks per CTA: channels <= 2048
constexpr int MAX_NB = 32;                  // images per cluster
constexpr int POOL_THREADS = 512;
constexpr int MMA_WARP = POOL_THREADS / 32;
constexpr int THREADS = POOL_THREADS + 32;
constexpr int LOADS = 16;                   // token rows a pool thread has in flight at once
constexpr int W_TILE = TN * 128;            // 128 classes x 64 channels, 16 KB
constexpr int PART_LD = MAX_NT * TN;        // partial logits: [MN][PART_LD] f32 over the weight tiles
constexpr int RED_BYTES = 16384;

// Shared-memory plan for MN image slots (the MMA's N).
template <int MN>
struct HL {
  static constexpr int B_TILE = MN * 128;               // MN images x 64 channels
  static constexpr int OFF_W = 0;
  static constexpr int OFF_B = MAX_NT * W_TILE;
  static constexpr int OFF_RED = OFF_B + MAX_KCH * B_TILE;
  static constexpr int OFF_BIAS = OFF_RED + RED_BYTES;
  static constexpr int OFF_BAR = OFF_BIAS + TN * 4;
  static constexpr int NBAR = 3 * MAX_KCH + 1;          // weights[k], pooled tile[k], MMA done[k], probe
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;
  static constexpr int TMEM_COLS = MAX_NT * MN;         // 128 or 256
  static_assert(MN == 16 || MN == 32, "image slots");
  static_assert(MN * PART_LD * 4 <= OFF_B, "partials fit the weight tiles");
  static_assert(SMEM <= 232448, "shared memory budget");
};
static_assert(CL * TN >= MAX_NT * TN, "every class tile has a reducing rank");

struct HeadArgs {
  const void* x;      // [B, HW, C]
  int64_t B;
  int HW, C, NC;
  int NB;             // images per cluster (<= MN)
  int KCH, NT;        // 64-channel chunks per CTA, class tiles
  float inv_hw;
  const void* bias;
  int bias_dt;
  void* out;          // [B, NC]
  void* pooled;       // [B, C] or null
  int* fault;
  uint32_t probe_ns;
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Every thread of every CTA in the cluster; release / acquire orders the
// shared-memory writes before it against the peers' reads after it.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t peer_addr(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}

__device__ __forceinline__ float4 ld_peer_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// 2-D TMA tile load into this CTA's shared memory, completing on ``bar``.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void pool_bar_sync() { asm volatile("bar.sync 1, %0;" ::"n"(POOL_THREADS) : "memory"); }

// 16-byte streaming load (the feature maps are read once).
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// acc[e] += the EPV elements of one 16-byte vector.
template <typename TX, bool BF16>
__device__ __forceinline__ void add_vec(float* acc, uint4 u) {
  if constexpr (sizeof(TX) == 4) {
    acc[0] += __uint_as_float(u.x);
    acc[1] += __uint_as_float(u.y);
    acc[2] += __uint_as_float(u.z);
    acc[3] += __uint_as_float(u.w);
  } else {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = unpack2<BF16>(w[i]);
      acc[2 * i] += f.x;
      acc[2 * i + 1] += f.y;
    }
  }
}

// Weight conversion to the compute type (row-major [NC, C]), for f32 weights.
template <typename T16>
__global__ void head_wprep_kernel(const float* __restrict__ w, int64_t n, T16* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = Elem<T16>::from(w[i]);
}

template <typename TX, bool BF16, int MN>
__global__ void __cluster_dims__(CL, 1, 1) __launch_bounds__(THREADS, 1)
    head_kernel(const __grid_constant__ CUtensorMap wmap, HeadArgs a) {
  using T16 = std::conditional_t<BF16, __nv_bfloat16, __half>;
  using L = HL<MN>;
  constexpr int EPV = 16 / (int)sizeof(TX);      // elements per 16-byte vector
  constexpr int VPR = 64 / EPV;                  // vectors per 64-channel chunk of a token row
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::OFF_BAR);
  uint64_t* bar_w = bars;
  uint64_t* bar_b = bars + MAX_KCH;
  uint64_t* bar_m = bars + 2 * MAX_KCH;
  uint64_t* bar_probe = bars + 3 * MAX_KCH;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + L::NBAR);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* bias_s = reinterpret_cast<float*>(sm + L::OFF_BIAS);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_rank();
  const int NB = a.NB;
  const int64_t img0 = (int64_t)(blockIdx.x / CL) * NB;
  const int ch0 = (int)rank * (a.C / CL);

  if (tid == 0) {
    for (int k = 0; k < MAX_KCH; ++k) {
      mbar_init(bar_w + k, 1);
      mbar_init(bar_b + k, POOL_THREADS);
      mbar_init(bar_m + k, 1);
    }
    mbar_init(bar_probe, 1);
    *abort = 0;
    fence_mbar_init();
    wait_probe(bar_probe, abort, a.probe_ns);
  }
  if (warp == MMA_WARP) tmem_alloc(tmem_holder, L::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_holder;
  // Only the setup's wait-timeout self-check can stop the pool: the pool
  // threads wait on nothing but each other, so all of them run the same
  // iterations (their named barrier needs every one).
  const bool live = !*abort;

  if (warp == MMA_WARP) {
    // One thread: the weight slices by TMA (one 64-channel chunk of every
    // class tile at a time, reusing the same tiles) and the MMAs.
    if (lane == 0 && live) {
      constexpr uint32_t ID = idesc_f16(TN, MN, BF16);
      const uint32_t sW = smem_u32(sm + L::OFF_W), sB = smem_u32(sm + L::OFF_B);
      auto load_w = [&](int kc) {
        mbar_arrive_expect_tx(bar_w + kc, (uint32_t)(a.NT * W_TILE));
        for (int j = 0; j < a.NT; ++j)
          tma_load_2d(sm + L::OFF_W + j * W_TILE, &wmap, ch0 + 64 * kc, TN * j, bar_w + kc);
      };
      load_w(0);
      for (int kc = 0; kc < a.KCH; ++kc) {
        if (!mbar_wait(bar_w + kc, 0, abort) || !mbar_wait(bar_b + kc, 0, abort)) break;
        tc_fence_after();
        for (int j = 0; j < a.NT; ++j)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16(tbase + j * MN, sdesc_sw128(sw128_kstep(sW + j * W_TILE, kk, TN)),
                     sdesc_sw128(sw128_kstep(sB + kc * L::B_TILE, kk, MN)), ID, (kc > 0 || kk > 0) ? 1u : 0u);
        umma_commit(bar_m + kc);
        if (kc + 1 < a.KCH) {
          // the tiles are reused: the next slice lands once these MMAs are done
          if (!mbar_wait(bar_m + kc, 0, abort)) break;
          load_w(kc + 1);
        }
      }
    }
    __syncwarp();
  } else {
    // Bias of this rank's classes, rounded to the compute type as autocast
    // casts it (read while the pool's loads are in flight).
    if (tid < TN) {
      const int n = (int)rank * TN + tid;
      float bv = 0.f;
      if (a.bias && n < a.NC) {
        if (a.bias_dt == OW_DTYPE_F32) bv = reinterpret_cast<const float*>(a.bias)[n];
        else if (a.bias_dt == OW_DTYPE_BF16) bv = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.bias)[n]);
        else bv = __half2float(reinterpret_cast<const __half*>(a.bias)[n]);
        bv = Elem<T16>::to_f(Elem<T16>::from(bv));
      }
      bias_s[tid] = bv;
    }
    // Pool: thread (sp, im, v) sums tokens [tk0, tk1) of vector v of image
    // im; SPLIT token ranges per (image, vector) use the pool threads.
    const int slots = NB * VPR, split = POOL_THREADS / slots;
    const int slot = tid % slots, v = slot % VPR, im = slot / VPR, sp = tid / slots;
    const bool active = sp < split;
    const int64_t b = img0 + im;
    const int tk0 = active ? (int)((int64_t)a.HW * sp / split) : 0;
    const int tk1 = active ? (int)((int64_t)a.HW * (sp + 1) / split) : 0;
    float* red = reinterpret_cast<float*>(sm + L::OFF_RED);
    // image slots NB.. of the MMA's N are zero
    if (NB < MN && live)
      for (int i = tid; i < a.KCH * MN * 8; i += POOL_THREADS) {
        const int row = (i >> 3) % MN;
        if (row >= NB) *reinterpret_cast<uint4*>(sm + L::OFF_B + i * 16) = make_uint4(0, 0, 0, 0);
      }
    for (int kc = 0; kc < (live ? a.KCH : 0); ++kc) {
      float acc[EPV];
#pragma unroll
      for (int e = 0; e < EPV; ++e) acc[e] = 0.f;
      const int c = ch0 + 64 * kc + v * EPV;
      if (b < a.B) {
        // batches of LOADS rows, all in flight together (rows past tk1 are not read)
        const TX* src = reinterpret_cast<const TX*>(a.x) + ((int64_t)b * a.HW) * a.C + c;
        for (int t0 = tk0; t0 < tk1; t0 += LOADS) {
          uint4 u[LOADS];
#pragma unroll
          for (int i = 0; i < LOADS; ++i)
            u[i] = t0 + i < tk1 ? ld_stream16(src + (int64_t)(t0 + i) * a.C) : make_uint4(0, 0, 0, 0);
#pragma unroll
          for (int i = 0; i < LOADS; ++i) add_vec<TX, BF16>(acc, u[i]);
        }
      }
      if (split > 1) {
        if (active && sp > 0)
#pragma unroll
          for (int e = 0; e < EPV; ++e) red[((sp - 1) * slots + slot) * EPV + e] = acc[e];
        pool_bar_sync();
        if (sp == 0)
          for (int s = 1; s < split; ++s)
#pragma unroll
            for (int e = 0; e < EPV; ++e) acc[e] += red[((s - 1) * slots + slot) * EPV + e];
        pool_bar_sync();
      }
      if (sp == 0) {
        uint32_t pk[EPV / 2];
#pragma unroll
        for (int e = 0; e < EPV / 2; ++e)
          pk[e] = b < a.B ? pack2<BF16>(acc[2 * e] * a.inv_hw, acc[2 * e + 1] * a.inv_hw) : 0u;
        unsigned char* dst = sm + L::OFF_B + kc * L::B_TILE + sw128_off(im, v * EPV, MN);
        if constexpr (EPV == 8) {
          const uint4 o = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          *reinterpret_cast<uint4*>(dst) = o;
          if (a.pooled && b < a.B) *reinterpret_cast<uint4*>(reinterpret_cast<T16*>(a.pooled) + b * a.C + c) = o;
        } else {
          const uint2 o = make_uint2(pk[0], pk[1]);
          *reinterpret_cast<uint2*>(dst) = o;
          if (a.pooled && b < a.B) *reinterpret_cast<uint2*>(reinterpret_cast<T16*>(a.pooled) + b * a.C + c) = o;
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(bar_b + kc);
    }
    // Partial logits of this channel slice: TMEM -> [image][class] f32 over
    // the weight tiles (the MMAs that read them are done).
    const bool ok = mbar_wait(bar_m + a.KCH - 1, 0, abort);
    tc_fence_after();
    if (ok) {
      float* part = reinterpret_cast<float*>(sm + L::OFF_W);
      const int q = warp & 3;
      for (int j = warp >> 2; j < a.NT; j += POOL_THREADS / 128) {
        uint32_t r[MN];
        tmem_ld_cols<MN>(tbase + ((uint32_t)(q * 32) << 16) + (uint32_t)(j * MN), r);
        tmem_ld_wait();
        const int cls = j * TN + q * 32 + lane;
#pragma unroll
        for (int i = 0; i < MN; ++i) part[i * PART_LD + cls] = __uint_as_float(r[i]);
      }
    }
    tc_fence_before();
  }

  __syncwarp();
  cluster_sync();
  // Rank r sums classes [128 r, 128 r + 128) over the eight slices in rank
  // order, adds the bias and stores the logits.
  if (tid < POOL_THREADS && (int)rank * TN < a.NC) {
    const uint32_t part0 = smem_u32(sm + L::OFF_W);
    T16* out = reinterpret_cast<T16*>(a.out);
    for (int idx = tid; idx < NB * (TN / 4); idx += POOL_THREADS) {
      const int im = idx / (TN / 4), cl = 4 * (idx % (TN / 4)), cls = (int)rank * TN + cl;
      const int64_t b = img0 + im;
      if (b >= a.B || cls >= a.NC) continue;
      const uint32_t off = part0 + (uint32_t)((im * PART_LD + cls) * 4);
      float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int r = 0; r < CL; ++r) {
        const float4 p = ld_peer_f4(peer_addr(off, (uint32_t)r));
        s.x += p.x;
        s.y += p.y;
        s.z += p.z;
        s.w += p.w;
      }
      const float sv[4] = {s.x, s.y, s.z, s.w};
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (cls + e < a.NC) out[b * a.NC + cls + e] = Elem<T16>::from(sv[e] + bias_s[cl + e]);
    }
  }
  // No CTA leaves while a peer may still read its partials.
  __syncwarp();
  cluster_sync();

  __syncthreads();
  report_abort(abort, a.fault);
  if (*abort)
    for (int i = 0; i < 1000; ++i) __nanosleep(1000);
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tbase, L::TMEM_COLS);
  }
}

bool is16(int dt) { return dt == OW_DTYPE_BF16 || dt == OW_DTYPE_F16; }

int head_check(const ow_pool_head_t* a, const char** why) {
  auto no = [&](const char* m) {
    if (why) *why = m;
    return OW_ERR_UNSUPPORTED;
  };
  if (!a) return no("args is NULL");
  if (!is16(a->compute_dtype)) return no("compute dtype must be bfloat16 or float16");
  if (a->batch <= 0 || a->tokens <= 0 || a->channels <= 0 || a->classes <= 0)
    return no("batch, tokens, channels and classes must be positive");
  if (a->x_dtype != OW_DTYPE_F32 && a->x_dtype != a->compute_dtype)
    return no("x dtype must be float32 or the compute dtype");
  if (a->w_dtype != OW_DTYPE_F32 && a->w_dtype != a->compute_dtype)
    return no("weight dtype must be float32 or the compute dtype");
  if (a->bias && a->bias_dtype != OW_DTYPE_F32 && !is16(a->bias_dtype))
    return no("bias dtype must be float32, bfloat16 or float16");
  if (a->channels % (CL * 64) || a->channels > CL * 64 * MAX_KCH)
    return no("channels must be a multiple of 512, at most 2048");
  if (a->classes > MAX_NT * TN) return no("classes must be at most 1024");
  if ((int64_t)a->batch * a->tokens * a->channels >= (1LL << 40)) return no("x too large");
  return OW_OK;
}

// Clusters of the head kernel that fit on the current device at once
// (asked once per device; every variant keeps one CTA per SM); 0 if the
// runtime cannot tell.
template <typename Kern>
int max_clusters(Kern kern, int smem) {
  static std::mutex mu;
  static int cache[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  std::lock_guard<std::mutex> lk(mu);
  if (cache[dev] == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(CL);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = (size_t)smem;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, (const void*)kern, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      return 0;
    }
    cache[dev] = n;
  }
  return cache[dev];
}

}  // namespace
}  // namespace ow

using namespace ow;

extern "C" {

size_t ow_pool_head_workspace_size(const ow_pool_head_t* a) {
  if (head_check(a, nullptr) != OW_OK) return 0;
  return (a->w_dtype == a->compute_dtype ? 0 : (size_t)a->classes * a->channels * 2) + 256;
}

int ow_pool_head_fwd(const ow_pool_head_t* a, void* stream) {
  clear_error();
  const char* why = nullptr;
  if (head_check(a, &why) != OW_OK) {
    set_error("ow_pool_head_fwd: %s", why);
    return OW_ERR_UNSUPPORTED;
  }
  OW_CHECK_ARG(a->x && a->weight && a->out, "ow_pool_head_fwd: a pointer is NULL");
  OW_CHECK_ARG((uintptr_t)a->x % 16 == 0 && (uintptr_t)a->weight % 16 == 0 && (uintptr_t)a->out % 2 == 0 &&
                   (uintptr_t)a->pooled % 16 == 0,
               "ow_pool_head_fwd: x, weight and pooled must be 16-byte aligned");
  const size_t need = ow_pool_head_workspace_size(a);
  if (!a->workspace || a->workspace_bytes < need) {
    set_error("ow_pool_head_fwd needs %zu workspace bytes, got %zu", need, a->workspace_bytes);
    return OW_ERR_WORKSPACE;
  }
  cudaStream_t st = (cudaStream_t)stream;
  const bool bf = a->compute_dtype == OW_DTYPE_BF16;
  const int sms = device_sm_count();
  HeadArgs k{};
  k.x = a->x;
  k.B = a->batch;
  k.HW = a->tokens;
  k.C = a->channels;
  k.NC = a->classes;
  k.KCH = a->channels / (CL * 64);
  k.NT = (a->classes + TN - 1) / TN;
  k.inv_hw = 1.0f / (float)a->tokens;
  k.bias = a->bias;
  k.bias_dt = a->bias_dtype;
  k.out = a->out;
  k.pooled = a->pooled;
  OW_RETURN_IF(fault_word(&k.fault));
  k.probe_ns = wait_probe_ns();

  const void* w16 = a->weight;
  if (a->w_dtype != a->compute_dtype) {
    unsigned char* img = (unsigned char*)(((uintptr_t)a->workspace + 255) & ~(uintptr_t)255);
    const int64_t n = (int64_t)a->classes * a->channels;
    const int pg = (int)std::min<int64_t>((n + 255) / 256, (int64_t)sms * 8);
    if (bf) launch(head_wprep_kernel<__nv_bfloat16>, pg, 256, 0, st, (const float*)a->weight, n, (__nv_bfloat16*)img);
    else launch(head_wprep_kernel<__half>, pg, 256, 0, st, (const float*)a->weight, n, (__half*)img);
    OW_CHECK_LAUNCH("head_wprep_kernel");
    w16 = img;
  }
  CUtensorMap map;
  const uint64_t dims[2] = {(uint64_t)a->channels, (uint64_t)a->classes};
  const uint64_t strides[1] = {(uint64_t)a->channels * 2};
  const uint32_t box[2] = {64, TN};
  OW_RETURN_IF(encode_tiled_map(&map, bf, 2, w16, dims, strides, box, "pool head"));

  auto setattr = [&](auto kern, int smem) -> int {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) {
      set_error("pool head: cannot reserve %d bytes of shared memory: %s", smem, cudaGetErrorString(e));
      return OW_ERR_CUDA;
    }
    return OW_OK;
  };
  auto run = [&](auto k16, auto k32) -> int {
    OW_RETURN_IF(setattr(k16, HL<16>::SMEM));
    OW_RETURN_IF(setattr(k32, HL<32>::SMEM));
    // One wave: the batch spread over the clusters that fit at once (at
    // least 8 images each), up to 32 images per cluster.
    int fit = max_clusters(k32, HL<32>::SMEM);
    if (fit <= 0) fit = std::max(1, sms / CL);
    int64_t ncl = std::min<int64_t>(fit, (k.B + 7) / 8);
    int64_t nb = std::min<int64_t>((k.B + ncl - 1) / ncl, MAX_NB);
    ncl = (k.B + nb - 1) / nb;
    if (ncl * CL >= (1LL << 31)) {
      set_error("ow_pool_head_fwd: batch too large");
      return OW_ERR_UNSUPPORTED;
    }
    k.NB = (int)nb;
    const int grid = (int)(ncl * CL);
    if (nb <= 16) launch(k16, grid, THREADS, HL<16>::SMEM, st, map, k);
    else launch(k32, grid, THREADS, HL<32>::SMEM, st, map, k);
    OW_CHECK_LAUNCH("head_kernel");
    return OW_OK;
  };
  if (a->x_dtype == OW_DTYPE_F32) {
    if (bf) return run(head_kernel<float, true, 16>, head_kernel<float, true, 32>);
    return run(head_kernel<float, false, 16>, head_kernel<float, false, 32>);
  }
  if (bf) return run(head_kernel<__nv_bfloat16, true, 16>, head_kernel<__nv_bfloat16, true, 32>);
  return run(head_kernel<__half, false, 16>, head_kernel<__half, false, 32>);
}

}  // extern "C"
