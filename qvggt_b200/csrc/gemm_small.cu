// Small-M tcgen05 GEMM (1 <= M <= 256 rows, e.g. the camera-head trunk whose
// linears see one token per frame): C[M, N] = A[M, K] . B[N, K]^T, computed as
// C^T = B . A^T so that 128 output channels form the MMA's 128-row operand and
// the M rows, padded to MT = 16..256, form its N dimension.  This is the role
// of the reference's small-M kernel gemm_w4a16_T1 (gemm_cuda.cu:312-751, with a
// global-memory semaphore for its split-K = 2 at M <= 32).
//
// Split-K on a thread-block cluster: the CTAs of one cluster share a
// 128-channel tile and each owns a contiguous K range, so N/128 tiles x splits
// fills the GPU even when N/128 is far below the SM count.  Every CTA issues
// all of its loads up front (the stage ring is as deep as its K range for the
// shapes of the camera trunk), parks its fp32 partial tile in its own shared
// memory, and after a cluster barrier each CTA reduces a slice of the tile by
// reading every peer's partial through distributed shared memory in rank
// order (deterministic), applies the fused epilogue (bias, GELU or LayerScale
// residual, same fp16 rounding points as the large kernel) and stores it.  No
// global workspace, atomics or extra launches.
//
// Operand modes: B_W4 (AWQ int4, dequantised by 4 warps into the K-major
// 128-byte-swizzled layout) and B_F16 (dense fp16 weight via TMA).
#include <cstdlib>

#include "gemm_common.cuh"
#include "gemm_sm100.cuh"
#include "host.hpp"

namespace qv {
namespace {

constexpr int SBN = 128;         // output channels per CTA (the MMA's M)
constexpr int MAX_SPLITS = 8;    // portable cluster size

template <int MT, int MODE>
struct SCfg {
  static constexpr int NS = MT <= 32 ? 8 : (MT <= 128 ? 6 : 4);
  static constexpr int ND = (mode_is_w4(MODE)) ? 2 : 0;
  static constexpr int X_BYTES = MT * 128;                                 // MT rows x 64 fp16
  static constexpr int W_BYTES = SBN * 128;                                // fp16 weight tile
  static constexpr int BQ_BYTES = (mode_is_w4(MODE)) ? (SBN / 4) * 128 : 0;     // packed int4 tile
  static constexpr int SZ_BYTES = (mode_is_w4(MODE)) ? 2 * SBN * 2 : 0;         // scales + zeros
  static constexpr int NUM_DQ_WARPS = (mode_is_w4(MODE)) ? SBN / 32 : 0;
  static constexpr int THREADS = 256 + NUM_DQ_WARPS * 32;
  static constexpr int OFF_X = 0;
  static constexpr int OFF_W = OFF_X + NS * X_BYTES;                       // dense W stages or packed stages
  static constexpr int OFF_D = OFF_W + NS * ((mode_is_w4(MODE)) ? BQ_BYTES : W_BYTES);
  static constexpr int OFF_SZ = OFF_D + ND * W_BYTES;
  static constexpr int OFF_BAR = ((OFF_SZ + NS * SZ_BYTES) + 15) / 16 * 16;
  static constexpr int NUM_BARS = 4 * NS + 2 * ND + 2;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int SMEM = OFF_MISC + 16 + 1024;
  static constexpr uint32_t TMEM_COLS = MT < 32 ? 32 : MT;
  // The fp32 partial tile [MT][128] reuses the X / W stage region.
  static constexpr int RED_BYTES = MT * SBN * 4;
  static_assert(RED_BYTES <= OFF_D, "partial tile must fit in the stage region");
};

struct SmallArgs {
  gemmk::GemmArgs g;
  int splits;        // CTAs per cluster = K ranges per channel tile
  int kb_per_split;
};

using namespace gemmk;

// The W4A16 / fp16 epilogue of one element (same rounding points as the large
// kernel's epilogue16): y = half(half(acc) + bias), then GELU or
// resid + half(y * gamma).  B_W4BF: bf16(acc) + bias, rounded to bf16 by the
// store.
template <int MODE>
__device__ __forceinline__ float small_final(const GemmArgs& g, float y, float b, int m, int n) {
  if constexpr (MODE == B_W4BF) return g.bias != nullptr ? round_bf16(y) + b : y;
  y = round_f16(y);
  if (g.bias != nullptr) y = round_f16(y + b);
  if (g.epi == EPI_GELU) {
    y = gelu_erf(y);
  } else if (g.epi == EPI_RESID) {
    y = __half2float(g.resid[(long long)m * g.ldr + n]) + round_f16(y * __half2float(g.gamma[n]));
  }
  return y;
}

template <int MT, int MODE>
__global__ void __launch_bounds__(SCfg<MT, MODE>::THREADS)
    gemm_small_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                      const __grid_constant__ CUtensorMap tmS, const __grid_constant__ CUtensorMap tmZ, SmallArgs sa) {
  using C = SCfg<MT, MODE>;
  const GemmArgs& g = sa.g;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* full_a = bars;                 // [NS] TMA -> MMA (X, and W for B_F16)
  uint64_t* empty_a = bars + C::NS;        // [NS] MMA -> TMA
  uint64_t* full_b = bars + 2 * C::NS;     // [NS] TMA -> dequant (B_W4)
  uint64_t* empty_b = bars + 3 * C::NS;    // [NS] dequant -> TMA (B_W4)
  uint64_t* full_d = bars + 4 * C::NS;     // [ND] dequant -> MMA
  uint64_t* empty_d = full_d + C::ND;      // [ND] MMA -> dequant
  uint64_t* tmem_full = empty_d + C::ND;   // MMA -> epilogue
  uint64_t* drain_bar = tmem_full + 1;     // MMA drain on abort
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);
  float* red = reinterpret_cast<float*>(smem + C::OFF_X);  // [MT][128] partial tile (after the main loop)

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int split = sa.splits > 1 ? (int)cluster_ctarank() : 0;
  const int n_blk = blockIdx.x / sa.splits;
  const int kb0 = split * sa.kb_per_split;
  const int kb1 = min(g.num_kb, kb0 + sa.kb_per_split);
  const int nkb = kb1 - kb0;  // >= 1 by construction of the plan

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::NS; ++i) {
      mbar_init(&full_a[i], 1);
      mbar_init(&empty_a[i], 1);
      mbar_init(&full_b[i], 1);
      mbar_init(&empty_b[i], C::NUM_DQ_WARPS > 0 ? C::NUM_DQ_WARPS : 1);
    }
    for (int i = 0; i < C::ND; ++i) {
      mbar_init(&full_d[i], C::NUM_DQ_WARPS);
      mbar_init(&empty_d[i], 1);
    }
    mbar_init(tmem_full, 1);
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
    if constexpr (mode_is_w4(MODE)) {
      tma_prefetch_desc(&tmS);
      tma_prefetch_desc(&tmZ);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // no global memory touched so far: wait for the previous kernel in the
  // stream only now (programmatic dependent launch)
  pdl_wait();
  pdl_trigger();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (; it < nkb; ++it) {
        const int kb = kb0 + it;
        const int s = it % C::NS;
        const uint32_t ph = (it / C::NS) & 1;
        if (!mbar_wait(&empty_a[s], ph ^ 1, abort_flag, g.ctl, ST_TIMEOUT_TMA_EMPTY)) { ok = false; break; }
        uint8_t* sx = smem + C::OFF_X + s * C::X_BYTES;
        if constexpr (mode_is_w4(MODE)) {
          mbar_arrive_expect_tx(&full_a[s], C::X_BYTES);
          tma_load_2d(sx, &tmX, &full_a[s], kb * 64, 0);
          if (!mbar_wait(&empty_b[s], ph ^ 1, abort_flag, g.ctl, ST_TIMEOUT_TMA_EMPTY)) { ++it; ok = false; break; }
          uint8_t* sq = smem + C::OFF_W + s * C::BQ_BYTES;
          uint8_t* ssz = smem + C::OFF_SZ + s * C::SZ_BYTES;
          const int grp = (kb * 64) / g.group_size;
          mbar_arrive_expect_tx(&full_b[s], C::BQ_BYTES + C::SZ_BYTES);
          tma_load_2d(sq, &tmW, &full_b[s], kb * 64, n_blk * (SBN / 4));
          tma_load_2d(ssz, &tmS, &full_b[s], n_blk * SBN, grp);
          tma_load_2d(ssz + SBN * 2, &tmZ, &full_b[s], n_blk * SBN, grp);
        } else {
          uint8_t* sw = smem + C::OFF_W + s * C::W_BYTES;
          mbar_arrive_expect_tx(&full_a[s], C::X_BYTES + C::W_BYTES);
          tma_load_2d(sx, &tmX, &full_a[s], kb * 64, 0);
          tma_load_2d(sw, &tmW, &full_a[s], kb * 64, n_blk * SBN);
        }
      }
      if (!ok) {
        // Drain: wait (bounded) for every load already issued to land.
        const int issued = it;
        for (int s = 0; s < C::NS; ++s) {
          const int cnt = issued > s ? (issued - 1 - s) / C::NS + 1 : 0;
          if (cnt == 0) continue;
          mbar_wait_drain(&full_a[s], (cnt - 1) & 1, 200000000ull);
          if constexpr (mode_is_w4(MODE)) mbar_wait_drain(&full_b[s], (cnt - 1) & 1, 200000000ull);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(SBN, MT, false, false, MODE == B_W4BF);
      bool ok = true;
      for (int it = 0; it < nkb; ++it) {
        const int s = it % C::NS;
        const uint32_t ph = (it / C::NS) & 1;
        if (!mbar_wait(&full_a[s], ph, abort_flag, g.ctl, ST_TIMEOUT_FULL)) { ok = false; break; }
        const uint8_t* sw;
        int d = 0;
        if constexpr (mode_is_w4(MODE)) {
          d = it % C::ND;
          const uint32_t dph = (it / C::ND) & 1;
          if (!mbar_wait(&full_d[d], dph, abort_flag, g.ctl, ST_TIMEOUT_DEQ)) { ok = false; break; }
          sw = smem + C::OFF_D + d * C::W_BYTES;
        } else {
          sw = smem + C::OFF_W + s * C::W_BYTES;
        }
        tc_fence_after();
        const uint32_t w_addr = smem_u32(sw);
        const uint32_t x_addr = smem_u32(smem + C::OFF_X + s * C::X_BYTES);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_f16_ss(tmem_base, sdesc_sw128(w_addr + k * 32), sdesc_sw128(x_addr + k * 32), idesc, (it | k) != 0);
        tc_commit(&empty_a[s]);
        if constexpr (mode_is_w4(MODE)) tc_commit(&empty_d[d]);
      }
      if (ok) {
        tc_commit(tmem_full);
      } else {
        tc_commit(drain_bar);
        mbar_wait_drain(drain_bar, 0, 200000000ull);
      }
    }
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------------------ epilogue
    // TMEM lane = output channel, column = row of A.  The tmem_full commit
    // also means every MMA (hence every stage read) is complete, so the stage
    // region is free for the partial tile.
    const int q = warp - 4;
    const int nl = q * 32 + lane;  // channel within the tile
    const int n = n_blk * SBN + nl;
    if (mbar_wait_warp(tmem_full, 0, abort_flag, g.ctl, ST_TIMEOUT_TMEM)) {
      tc_fence_after();
      float b = 0.f;
      if (sa.splits == 1 && g.bias != nullptr)
        b = MODE == B_W4BF ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(g.bias)[n])
                           : __half2float(g.bias[n]);
#pragma unroll 1
      for (int c = 0; c < MT / 16 && c * 16 < g.M; ++c) {
        uint32_t r[16];
        tmem_ld16(tmem_addr(tmem_base, q * 32, c * 16), r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = c * 16 + j;
          const float acc = __uint_as_float(r[j]);
          if (sa.splits > 1)
            red[m * SBN + nl] = acc;
          else if (m < g.M && MODE == B_W4BF)
            reinterpret_cast<__nv_bfloat16*>(g.out)[(long long)m * g.ldo + n] =
                __float2bfloat16_rn(small_final<MODE>(g, acc, b, m, n));
          else if (m < g.M)
            g.out[(long long)m * g.ldo + n] = __float2half_rn(small_final<MODE>(g, acc, b, m, n));
        }
      }
    }
  } else if (warp >= 8) {
    // ------------------------------------------------------------ dequantisation
    if constexpr (mode_is_w4(MODE)) {
      const int n = threadIdx.x - 256;  // channel within the tile
      const int grow = n >> 2;          // packed row within the tile
      const int ci = n & 3;             // channel within the packed row
      for (int it = 0; it < nkb; ++it) {
        const int s = it % C::NS;
        const uint32_t ph = (it / C::NS) & 1;
        if (!mbar_wait_warp(&full_b[s], ph, abort_flag, g.ctl, ST_TIMEOUT_FULL)) break;
        const uint8_t* sq = smem + C::OFF_W + s * C::BQ_BYTES + grow * 128;
        const uint16_t* ssz = reinterpret_cast<const uint16_t*>(smem + C::OFF_SZ + s * C::SZ_BYTES);
        uint32_t x0[4], x1[4];
        *reinterpret_cast<uint4*>(x0) = *reinterpret_cast<const uint4*>(sq + (((2 * ci) ^ (grow & 7)) * 16));
        *reinterpret_cast<uint4*>(x1) = *reinterpret_cast<const uint4*>(sq + (((2 * ci + 1) ^ (grow & 7)) * 16));
        const uint32_t s2 = dup16(ssz + n);
        const uint32_t z2 = dup16(ssz + SBN + n);
        // the stage is refilled by TMA once released: retire these reads first
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_b[s]);
        const int d = it % C::ND;
        const uint32_t dph = (it / C::ND) & 1;
        if (!mbar_wait_warp(&empty_d[d], dph ^ 1, abort_flag, g.ctl, ST_TIMEOUT_DEQ)) break;
        uint8_t* drow = smem + C::OFF_D + d * C::W_BYTES + n * 128;
        uint4 o[4];
        dequant_chunk<MODE == B_W4BF>(x0, s2, z2, o);
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) *reinterpret_cast<uint4*>(drow + ((qq ^ (n & 7)) * 16)) = o[qq];
        dequant_chunk<MODE == B_W4BF>(x1, s2, z2, o);
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) *reinterpret_cast<uint4*>(drow + (((4 + qq) ^ (n & 7)) * 16)) = o[qq];
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full_d[d]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
  if (sa.splits == 1) return;

  // ---------------------------------------------------------------- split-K reduction
  // Every thread of every CTA of the cluster reaches both cluster barriers,
  // also after an aborted (timed-out) main loop; the status word then reports
  // the failure and the values stored are not meaningful.
  cluster_sync();
  if (!*abort_flag) {
    const int units = g.M * (SBN / 4);  // float4 units of the tile, m-major
    const int u0 = (int)(((long long)units * split) / sa.splits);
    const int u1 = (int)(((long long)units * (split + 1)) / sa.splits);
    for (int u = u0 + (int)threadIdx.x; u < u1; u += blockDim.x) {
      const int m = u / (SBN / 4);
      const int c4 = u % (SBN / 4);
      const float* src = red + m * SBN + c4 * 4;
      float4 acc = ld_cluster_f4(mapa_shared(src, 0));
      for (int r = 1; r < sa.splits; ++r) {
        const float4 v = ld_cluster_f4(mapa_shared(src, (uint32_t)r));
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      const int n = n_blk * SBN + c4 * 4;
      float b[4] = {0.f, 0.f, 0.f, 0.f};
      if (g.bias != nullptr) {
        const uint2 bu = *reinterpret_cast<const uint2*>(g.bias + n);
        const float2 b01 = MODE == B_W4BF ? unpack_bf162(bu.x) : unpack_half2(bu.x);
        const float2 b23 = MODE == B_W4BF ? unpack_bf162(bu.y) : unpack_half2(bu.y);
        b[0] = b01.x; b[1] = b01.y; b[2] = b23.x; b[3] = b23.y;
      }
      const float y0 = small_final<MODE>(g, acc.x, b[0], m, n);
      const float y1 = small_final<MODE>(g, acc.y, b[1], m, n + 1);
      const float y2 = small_final<MODE>(g, acc.z, b[2], m, n + 2);
      const float y3 = small_final<MODE>(g, acc.w, b[3], m, n + 3);
      *reinterpret_cast<uint2*>(g.out + (long long)m * g.ldo + n) =
          MODE == B_W4BF ? make_uint2(pack_bf162(y0, y1), pack_bf162(y2, y3))
                         : make_uint2(pack_half2(y0, y1), pack_half2(y2, y3));
    }
  }
  // No CTA may exit (releasing its shared memory) while a peer still reads it.
  cluster_sync();
}

// Opts the kernel into its dynamic shared memory once per device.
template <int MT, int MODE>
int ensure_smem_attr() {
  static DeviceFlags attr_set;
  const DeviceInfo& di = device_info();
  if (SCfg<MT, MODE>::SMEM > di.max_smem_optin)
    return set_error(QVGGT_ERR_UNSUPPORTED, "gemm_small: %d B shared memory exceeds the device limit",
                     SCfg<MT, MODE>::SMEM);
  return ensure_smem(attr_set, gemm_small_kernel<MT, MODE>, SCfg<MT, MODE>::SMEM, "cudaFuncSetAttribute(gemm_small)");
}

// How many clusters of `splits` CTAs of this kernel the device holds at once
// (cached per device and cluster size; relaxed atomics: two threads that both
// find an entry empty both compute the same value).
template <int MT, int MODE>
int active_clusters(int splits) {
  static std::atomic<int> cache[kMaxDevices][MAX_SPLITS + 1];
  const DeviceInfo& di = device_info();
  std::atomic<int> dummy{0};
  std::atomic<int>& slot = (di.device >= 0 && di.device < kMaxDevices) ? cache[di.device][splits] : dummy;
  int c = slot.load(std::memory_order_relaxed);
  if (c == 0) {
    if (ensure_smem_attr<MT, MODE>()) return 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(splits * di.num_sms), 1, 1);
    cfg.blockDim = dim3(SCfg<MT, MODE>::THREADS, 1, 1);
    cfg.dynamicSmemBytes = SCfg<MT, MODE>::SMEM;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_small_kernel<MT, MODE>, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = -1;  // unknown: treated as "does not fit"
    }
    c = n;
    slot.store(c, std::memory_order_relaxed);
  }
  return c;
}

// B_W4BF plans as B_W4: the same shared memory, threads and tiles.
int plan_active_clusters(int mt, int mode, int splits) {
  const bool w4 = mode_is_w4(mode);
  switch (mt) {
    case 16: return w4 ? active_clusters<16, B_W4>(splits) : active_clusters<16, B_F16>(splits);
    case 32: return w4 ? active_clusters<32, B_W4>(splits) : active_clusters<32, B_F16>(splits);
    case 64: return w4 ? active_clusters<64, B_W4>(splits) : active_clusters<64, B_F16>(splits);
    case 128: return w4 ? active_clusters<128, B_W4>(splits) : active_clusters<128, B_F16>(splits);
    default: return w4 ? active_clusters<256, B_W4>(splits) : active_clusters<256, B_F16>(splits);
  }
}

int plan_smem(int mt, int mode) {
  const bool w4 = mode_is_w4(mode);
  switch (mt) {
    case 16: return w4 ? SCfg<16, B_W4>::SMEM : SCfg<16, B_F16>::SMEM;
    case 32: return w4 ? SCfg<32, B_W4>::SMEM : SCfg<32, B_F16>::SMEM;
    case 64: return w4 ? SCfg<64, B_W4>::SMEM : SCfg<64, B_F16>::SMEM;
    case 128: return w4 ? SCfg<128, B_W4>::SMEM : SCfg<128, B_F16>::SMEM;
    default: return w4 ? SCfg<256, B_W4>::SMEM : SCfg<256, B_F16>::SMEM;
  }
}

template <int MT, int MODE>
int launch_small(const GemmLaunch& L, const SmallPlan& P) {
  using C = SCfg<MT, MODE>;
  CUtensorMap tmX, tmW, tmS, tmZ;
  constexpr CUtensorMapDataType act_type =
      MODE == B_W4BF ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  int rc = tmap_2d(&tmX, act_type, L.a, L.K, L.M, L.lda * 2, 64, MT, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  if constexpr (mode_is_w4(MODE)) {
    rc = tmap_2d(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT16, L.b, L.K, L.N / 4, L.K * 2, 64, SBN / 4,
                 CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = tmap_2d(&tmS, act_type, L.scales, L.N, L.gpad, L.N * 2, SBN, 1,
                 CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    rc = tmap_2d(&tmZ, act_type, L.zeros, L.N, L.gpad, L.N * 2, SBN, 1,
                 CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  } else {
    rc = tmap_2d(&tmW, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, L.b, L.K, L.N, L.K * 2, 64, SBN, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    tmS = tmW;
    tmZ = tmW;
  }
  SmallArgs sa;
  GemmArgs& g = sa.g;
  g.M = (int)L.M;
  g.N = (int)L.N;
  g.K = (int)L.K;
  g.n_blocks = P.n_blocks;
  g.num_tiles = P.n_blocks * P.splits;
  g.num_kb = P.num_kb;
  g.group_size = L.group_size;
  g.epi = L.epi;
  g.bias = reinterpret_cast<const __half*>(L.bias);
  g.out = reinterpret_cast<__half*>(L.out);
  g.ldo = L.ldo;
  g.resid = reinterpret_cast<const __half*>(L.resid);
  g.ldr = L.ldr;
  g.gamma = reinterpret_cast<const __half*>(L.gamma);
  g.wscale = nullptr;
  g.ascale = nullptr;
  g.rope = L.rope;
  g.ctl = make_ctl();
  sa.splits = P.splits;
  sa.kb_per_split = P.kb_per_split;
  auto kfn = gemm_small_kernel<MT, MODE>;
  rc = ensure_smem_attr<MT, MODE>();
  if (rc) return rc;
  return check_cuda(launch_pdl(kfn, dim3((unsigned)(P.n_blocks * P.splits)), dim3(C::THREADS), C::SMEM, L.stream,
                               (unsigned)P.splits, tmX, tmW, tmS, tmZ, sa),
                    "gemm_small launch");
}

}  // namespace

int gemm_small_plan(int mode, long long M, long long N, long long K, int max_splits, SmallPlan* P) {
  if (mode != B_W4 && mode != B_F16 && mode != B_W4BF)
    return set_error(QVGGT_ERR_UNSUPPORTED, "gemm_small: mode %d", mode);
  if (M < 1 || M > 256) return set_error(QVGGT_ERR_UNSUPPORTED, "gemm_small: M=%lld must be in 1..256", M);
  if (N <= 0 || N % SBN) return set_error(QVGGT_ERR_UNSUPPORTED, "gemm_small: N=%lld must be a multiple of 128", N);
  if (K <= 0 || K % 64) return set_error(QVGGT_ERR_UNSUPPORTED, "gemm_small: K=%lld must be a multiple of 64", K);
  P->mt = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
  P->n_blocks = (int)(N / SBN);
  P->num_kb = (int)(K / 64);
  P->smem = plan_smem(P->mt, mode);
  int cap = max_splits > 0 && max_splits < MAX_SPLITS ? max_splits : MAX_SPLITS;
  if (cap > P->num_kb) cap = P->num_kb;
  // Measured on B200 at the camera-trunk shapes: per-CTA time grows with its
  // K range, so for tiles of <= 32 rows the most splits whose clusters fit in
  // two waves win (co-resident clusters from the occupancy query); taller
  // tiles (more shared memory, heavier reduction) keep to one wave.
  // QVGGT_SMALL_SPLITS=n forces n CTAs per cluster.
  static int forced = -1;
  if (forced < 0) {
    const char* e = getenv("QVGGT_SMALL_SPLITS");
    forced = e ? atoi(e) : 0;
  }
  int splits = 1;
  P->active_clusters = plan_active_clusters(P->mt, mode, 1);
  if (forced > 0) {
    splits = forced < cap ? forced : cap;
    P->active_clusters = plan_active_clusters(P->mt, mode, splits);
  } else {
    const int waves = P->mt <= 32 ? 2 : 1;
    for (int s = 2; s <= cap; ++s) {
      if (P->num_kb / s < 2) break;  // at least 2 k-blocks per CTA
      const int a = plan_active_clusters(P->mt, mode, s);
      if (a > 0 && (long long)a * waves >= P->n_blocks) {
        splits = s;
        P->active_clusters = a;
      }
    }
  }
  P->kb_per_split = (P->num_kb + splits - 1) / splits;
  P->splits = (P->num_kb + P->kb_per_split - 1) / P->kb_per_split;
  return QVGGT_OK;
}

int gemm_small_launch(const GemmLaunch& L, const SmallPlan& P) {
  if (L.mode != B_W4 && L.mode != B_F16 && L.mode != B_W4BF) return set_error(QVGGT_ERR_UNSUPPORTED, "gemm_small: mode");
  if (L.epi != EPI_STORE && L.epi != EPI_GELU && L.epi != EPI_RESID)
    return set_error(QVGGT_ERR_UNSUPPORTED, "gemm_small: epilogue %d", L.epi);
  if (L.mode == B_W4BF && L.epi != EPI_STORE)
    return set_error(QVGGT_ERR_UNSUPPORTED, "gemm_small: bf16 activations take the plain store epilogue only");
  if (!aligned16(L.a) || !aligned16(L.b) || !aligned16(L.out) || (L.bias && !aligned16(L.bias)))
    return set_error(QVGGT_ERR_ALIGN, "gemm_small: operands must be 16-byte aligned");
  if (L.lda % 8 || L.ldo % 8 || (L.resid && L.ldr % 8))
    return set_error(QVGGT_ERR_ALIGN, "gemm_small: strides must be multiples of 8 elements");
  if (mode_is_w4(L.mode)) {
    if (L.group_size <= 0 || L.group_size % 64 != 0 || L.K % L.group_size != 0)
      return set_error(QVGGT_ERR_UNSUPPORTED, "gemm_small: group_size=%d must be a multiple of 64 dividing K",
                       L.group_size);
    if (L.gpad < L.K / L.group_size) return set_error(QVGGT_ERR_INVALID, "gemm_small: scale table has too few groups");
    if (!aligned16(L.scales) || !aligned16(L.zeros)) return set_error(QVGGT_ERR_ALIGN, "gemm_small: scales not aligned");
  }
  if (L.epi == EPI_RESID && (!L.resid || !L.gamma)) return set_error(QVGGT_ERR_INVALID, "gemm_small: residual needs resid+gamma");
  if (P.splits < 1 || P.splits > MAX_SPLITS) return set_error(QVGGT_ERR_INVALID, "gemm_small: bad plan");
  if (L.mode == B_W4BF) {
    switch (P.mt) {
      case 16: return launch_small<16, B_W4BF>(L, P);
      case 32: return launch_small<32, B_W4BF>(L, P);
      case 64: return launch_small<64, B_W4BF>(L, P);
      case 128: return launch_small<128, B_W4BF>(L, P);
      case 256: return launch_small<256, B_W4BF>(L, P);
    }
    return set_error(QVGGT_ERR_INVALID, "gemm_small: bad plan");
  }
  const bool w4 = L.mode == B_W4;
  switch (P.mt) {
    case 16: return w4 ? launch_small<16, B_W4>(L, P) : launch_small<16, B_F16>(L, P);
    case 32: return w4 ? launch_small<32, B_W4>(L, P) : launch_small<32, B_F16>(L, P);
    case 64: return w4 ? launch_small<64, B_W4>(L, P) : launch_small<64, B_F16>(L, P);
    case 128: return w4 ? launch_small<128, B_W4>(L, P) : launch_small<128, B_F16>(L, P);
    case 256: return w4 ? launch_small<256, B_W4>(L, P) : launch_small<256, B_F16>(L, P);
  }
  return set_error(QVGGT_ERR_INVALID, "gemm_small: bad plan");
}

}  // namespace qv
