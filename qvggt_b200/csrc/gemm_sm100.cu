// Persistent tcgen05 GEMM for sm_100a: C[M, N] = A[M, K] . B[N, K]^T with a
// fused epilogue, in three operand modes:
//
//   B_W4  : A fp16, B = AWQ-packed int4 (qweight int16 [N/4, K]) with fp16
//           per-group scales / scaled zeros [Gpad, N].  TMA brings the packed
//           words and the group's scales into shared memory; dequantisation
//           warps turn them into fp16 in the 128-byte-swizzled K-major layout
//           the tensor core reads; fp32 accumulation in TMEM.
//   B_F16 : A fp16, B fp16 [N, K] (dense, e.g. the unquantised patch embed).
//   B_I8  : A int8 [M, K], B int8 [N, K], int32 accumulation in TMEM, and the
//           per-token x per-channel rescale epilogue of the reference W8A8 GEMM.
//
// Tile 128 x BN x (128 bytes of K), one CTA per SM, static persistent tile
// schedule (m-major so CTAs running together share A rows in L2), two TMEM
// accumulators so the epilogue of tile i overlaps the main loop of tile i+1.
//
// Warp roles: warp 0 = TMA producer, warp 1 = TMEM owner + MMA issuer,
// warps 4..7 = epilogue (TMEM lane quarters 0..3), warps 8.. = dequantisation
// (B_W4 only).  All inter-role waits are bounded (see common.cuh).
#include <atomic>

#include "gemm_common.cuh"

#include "gemm_sm100.cuh"
#include "host.hpp"

namespace qv {
namespace {

constexpr int BM = 128;
constexpr int KB_BYTES = 128;  // bytes of K per k-block (64 fp16 or 128 int8)

template <int BN, int MODE>
struct Cfg {
  static constexpr int NS = (mode_is_w4(MODE)) ? (BN == 256 ? 4 : 6) : (BN == 256 ? 4 : 6);
  static constexpr int ND = (mode_is_w4(MODE)) ? 3 : 0;
  static constexpr int A_BYTES = BM * KB_BYTES;                           // 16 KB
  static constexpr int B_BYTES = BN * KB_BYTES;                           // fp16/int8 operand tile
  static constexpr int BQ_BYTES = (mode_is_w4(MODE)) ? (BN / 4) * KB_BYTES : 0; // packed int4 tile
  static constexpr int SZ_BYTES = (mode_is_w4(MODE)) ? 2 * BN * 2 : 0;         // scales + zeros
  static constexpr int NUM_DQ_WARPS = (mode_is_w4(MODE)) ? BN / 32 : 0;
  static constexpr int THREADS = 256 + NUM_DQ_WARPS * 32;
  // shared memory carve-up (offsets from a 1024-aligned base)
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + NS * A_BYTES;                      // B_F16/B_I8 operand stages
  static constexpr int OFF_BQ = OFF_A + NS * A_BYTES;                     // B_W4 packed stages
  static constexpr int OFF_D = (mode_is_w4(MODE)) ? OFF_BQ + NS * BQ_BYTES : OFF_B + NS * B_BYTES;
  static constexpr int OFF_SZ = OFF_D + ND * B_BYTES;
  static constexpr int OFF_BAR = ((OFF_SZ + NS * SZ_BYTES) + 15) / 16 * 16;
  static constexpr int NUM_BARS = 4 * NS + 2 * ND + 4 + 1;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int SMEM = OFF_MISC + 16 + 1024;  // + alignment slack
  static constexpr uint32_t TMEM_COLS = 2 * BN <= 32 ? 32 : (2 * BN <= 64 ? 64 : (2 * BN <= 128 ? 128 : (2 * BN <= 256 ? 256 : 512)));
};

using namespace gemmk;

template <int BN, int MODE>
__global__ void __launch_bounds__(Cfg<BN, MODE>::THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmS, const __grid_constant__ CUtensorMap tmZ, GemmArgs g) {
  using C = Cfg<BN, MODE>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* full_a = bars;                 // [NS] TMA -> MMA (A, and B for dense modes)
  uint64_t* empty_a = bars + C::NS;        // [NS] MMA -> TMA
  uint64_t* full_b = bars + 2 * C::NS;     // [NS] TMA -> dequant (B_W4)
  uint64_t* empty_b = bars + 3 * C::NS;    // [NS] dequant -> TMA (B_W4)
  uint64_t* full_d = bars + 4 * C::NS;     // [ND] dequant -> MMA
  uint64_t* empty_d = full_d + C::ND;      // [ND] MMA -> dequant
  uint64_t* tmem_full = empty_d + C::ND;   // [2] MMA -> epilogue
  uint64_t* tmem_empty = tmem_full + 2;    // [2] epilogue -> MMA
  uint64_t* drain_bar = tmem_empty + 2;    // MMA drain on abort
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

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
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tmem_full[i], 1);
      mbar_init(&tmem_empty[i], 4);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
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

  const int num_kb = g.num_kb;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < g.num_tiles && ok; tile += gridDim.x) {
        const int m_blk = tile / g.n_blocks, n_blk = tile % g.n_blocks;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % C::NS;
          const uint32_t ph = (it / C::NS) & 1;
          if (!mbar_wait(&empty_a[s], ph ^ 1, abort_flag, g.ctl, ST_TIMEOUT_TMA_EMPTY)) { ok = false; break; }
          uint8_t* sa = smem + C::OFF_A + s * C::A_BYTES;
          if constexpr (mode_is_w4(MODE)) {
            mbar_arrive_expect_tx(&full_a[s], C::A_BYTES);
            tma_load_2d(sa, &tmA, &full_a[s], kb * 64, m_blk * BM);
            if (!mbar_wait(&empty_b[s], ph ^ 1, abort_flag, g.ctl, ST_TIMEOUT_TMA_EMPTY)) { ++it; ok = false; break; }
            uint8_t* sq = smem + C::OFF_BQ + s * C::BQ_BYTES;
            uint8_t* ssz = smem + C::OFF_SZ + s * C::SZ_BYTES;
            const int grp = (kb * 64) / g.group_size;
            mbar_arrive_expect_tx(&full_b[s], C::BQ_BYTES + C::SZ_BYTES);
            tma_load_2d(sq, &tmB, &full_b[s], kb * 64, n_blk * (BN / 4));
            tma_load_2d(ssz, &tmS, &full_b[s], n_blk * BN, grp);
            tma_load_2d(ssz + BN * 2, &tmZ, &full_b[s], n_blk * BN, grp);
          } else {
            uint8_t* sb = smem + C::OFF_B + s * C::B_BYTES;
            mbar_arrive_expect_tx(&full_a[s], C::A_BYTES + C::B_BYTES);
            tma_load_2d(sa, &tmA, &full_a[s], kb * KB_BYTES / (MODE == B_I8 ? 1 : 2), m_blk * BM);
            tma_load_2d(sb, &tmB, &full_a[s], kb * KB_BYTES / (MODE == B_I8 ? 1 : 2), n_blk * BN);
          }
        }
      }
      if (!ok) {
        // Drain: wait (bounded) for every load already issued to land.
        const uint32_t issued = it;
        for (int s = 0; s < C::NS; ++s) {
          const uint32_t cnt = issued > (uint32_t)s ? (issued - 1 - s) / C::NS + 1 : 0;
          if (cnt == 0) continue;
          mbar_wait_drain(&full_a[s], (cnt - 1) & 1, 200000000ull);
          if constexpr (mode_is_w4(MODE)) mbar_wait_drain(&full_b[s], (cnt - 1) & 1, 200000000ull);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = (MODE == B_I8) ? idesc_i8(BM, BN) : idesc_f16(BM, BN, false, false, MODE == B_W4BF);
      uint32_t it = 0;
      int t_local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < g.num_tiles && ok; tile += gridDim.x, ++t_local) {
        const int acc = t_local & 1;
        const uint32_t aph = (t_local >> 1) & 1;
        if (!mbar_wait(&tmem_empty[acc], aph ^ 1, abort_flag, g.ctl, ST_TIMEOUT_TMEM)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % C::NS;
          const uint32_t ph = (it / C::NS) & 1;
          if (!mbar_wait(&full_a[s], ph, abort_flag, g.ctl, ST_TIMEOUT_FULL)) { ok = false; break; }
          const uint8_t* sb;
          int d = 0;
          if constexpr (mode_is_w4(MODE)) {
            d = it % C::ND;
            const uint32_t dph = (it / C::ND) & 1;
            if (!mbar_wait(&full_d[d], dph, abort_flag, g.ctl, ST_TIMEOUT_DEQ)) { ok = false; break; }
            sb = smem + C::OFF_D + d * C::B_BYTES;
          } else {
            sb = smem + C::OFF_B + s * C::B_BYTES;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + C::OFF_A + s * C::A_BYTES);
          const uint32_t b_addr = smem_u32(sb);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t ad = sdesc_sw128(a_addr + k * 32);
            const uint64_t bd = sdesc_sw128(b_addr + k * 32);
            if constexpr (MODE == B_I8)
              mma_i8_ss(d_tmem, ad, bd, idesc, (kb | k) != 0);
            else
              mma_f16_ss(d_tmem, ad, bd, idesc, (kb | k) != 0);
          }
          tc_commit(&empty_a[s]);
          if constexpr (mode_is_w4(MODE)) tc_commit(&empty_d[d]);
        }
        if (!ok) break;
        tc_commit(&tmem_full[acc]);
      }
      if (!ok) {
        tc_commit(drain_bar);
        mbar_wait_drain(drain_bar, 0, 200000000ull);
      }
    }
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------------------ epilogue
    const int q = warp - 4;  // TMEM lane quarter
    int t_local = 0;
    for (int tile = blockIdx.x; tile < g.num_tiles; tile += gridDim.x, ++t_local) {
      const int m_blk = tile / g.n_blocks, n_blk = tile % g.n_blocks;
      const int acc = t_local & 1;
      const uint32_t aph = (t_local >> 1) & 1;
      if (!mbar_wait_warp(&tmem_full[acc], aph, abort_flag, g.ctl, ST_TIMEOUT_TMEM)) break;
      tc_fence_after();
      const int row = m_blk * BM + q * 32 + lane;
      const uint32_t tbase = tmem_addr(tmem_base, q * 32, acc * BN);
      if (MODE != B_I8 && MODE != B_W4BF && g.epi == EPI_QKV_ROPE) {
#pragma unroll 1
        for (int c = 0; c < BN / 64; ++c) {
          uint32_t r[64];
          tmem_ld32(tbase + c * 64, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
          tmem_ld32(tbase + c * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
          tmem_ld_wait();
          if (row < g.M) epilogue_qkv_head(g, row, n_blk * BN + c * 64, r);
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN / 16; ++c) {
          uint32_t r[16];
          tmem_ld16(tbase + c * 16, r);
          tmem_ld_wait();
          if (row < g.M) epilogue16<MODE>(g, row, n_blk * BN + c * 16, r);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tmem_empty[acc]);
    }
  } else if (warp >= 8) {
    // ------------------------------------------------------------ dequantisation
    if constexpr (mode_is_w4(MODE)) {
      const int n = threadIdx.x - 256;  // channel within the tile, 0..BN-1
      const int grow = n >> 2;          // packed row within the tile
      const int ci = n & 3;             // channel within the packed row
      uint32_t it = 0;
      for (int tile = blockIdx.x; tile < g.num_tiles; tile += gridDim.x) {
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % C::NS;
          const uint32_t ph = (it / C::NS) & 1;
          if (!mbar_wait_warp(&full_b[s], ph, abort_flag, g.ctl, ST_TIMEOUT_FULL)) { ok = false; break; }
          const uint8_t* sq = smem + C::OFF_BQ + s * C::BQ_BYTES + grow * 128;
          const uint16_t* ssz = reinterpret_cast<const uint16_t*>(smem + C::OFF_SZ + s * C::SZ_BYTES);
          uint32_t x0[4], x1[4];
          *reinterpret_cast<uint4*>(x0) = *reinterpret_cast<const uint4*>(sq + (((2 * ci) ^ (grow & 7)) * 16));
          *reinterpret_cast<uint4*>(x1) = *reinterpret_cast<const uint4*>(sq + (((2 * ci + 1) ^ (grow & 7)) * 16));
          const uint32_t s2 = dup16(ssz + n);
          const uint32_t z2 = dup16(ssz + BN + n);
          // the stage is refilled by TMA once released: retire these reads first
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty_b[s]);
          const int d = it % C::ND;
          const uint32_t dph = (it / C::ND) & 1;
          if (!mbar_wait_warp(&empty_d[d], dph ^ 1, abort_flag, g.ctl, ST_TIMEOUT_DEQ)) { ok = false; break; }
          uint8_t* drow = smem + C::OFF_D + d * C::B_BYTES + n * 128;
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
        if (!ok) break;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

template <int BN, int MODE>
int launch_gemm(const GemmLaunch& L) {
  using C = Cfg<BN, MODE>;
  const DeviceInfo& di = device_info();
  if (C::SMEM > di.max_smem_optin)
    return set_error(QVGGT_ERR_UNSUPPORTED, "gemm: %d B shared memory exceeds the device limit %d", C::SMEM,
                     di.max_smem_optin);
  CUtensorMap tmA, tmB, tmS, tmZ;
  int rc;
  constexpr CUtensorMapDataType act_type =
      MODE == B_W4BF ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  if constexpr (MODE == B_I8) {
    rc = tmap_2d(&tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, L.a, L.K, L.M, L.lda, 128, BM, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = tmap_2d(&tmB, CU_TENSOR_MAP_DATA_TYPE_UINT8, L.b, L.K, L.N, L.K, 128, BN, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    tmS = tmB;
    tmZ = tmB;
  } else {
    rc = tmap_2d(&tmA, act_type, L.a, L.K, L.M, L.lda * 2, 64, BM, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    if constexpr (mode_is_w4(MODE)) {
      rc = tmap_2d(&tmB, CU_TENSOR_MAP_DATA_TYPE_UINT16, L.b, L.K, L.N / 4, L.K * 2, 64, BN / 4,
                   CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc) return rc;
      rc = tmap_2d(&tmS, act_type, L.scales, L.N, L.gpad, L.N * 2, BN, 1,
                   CU_TENSOR_MAP_SWIZZLE_NONE);
      if (rc) return rc;
      rc = tmap_2d(&tmZ, act_type, L.zeros, L.N, L.gpad, L.N * 2, BN, 1,
                   CU_TENSOR_MAP_SWIZZLE_NONE);
      if (rc) return rc;
    } else {
      rc = tmap_2d(&tmB, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, L.b, L.K, L.N, L.K * 2, 64, BN, CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc) return rc;
      tmS = tmB;
      tmZ = tmB;
    }
  }
  GemmArgs g;
  g.M = (int)L.M;
  g.N = (int)L.N;
  g.K = (int)L.K;
  g.n_blocks = (int)(L.N / BN);
  const int m_blocks = (int)((L.M + BM - 1) / BM);
  g.num_tiles = m_blocks * g.n_blocks;
  g.num_kb = (int)(L.K * (MODE == B_I8 ? 1 : 2) / KB_BYTES);
  g.group_size = L.group_size;
  g.epi = L.epi;
  g.bias = reinterpret_cast<const __half*>(L.bias);
  g.out = reinterpret_cast<__half*>(L.out);
  g.ldo = L.ldo;
  g.resid = reinterpret_cast<const __half*>(L.resid);
  g.ldr = L.ldr;
  g.gamma = reinterpret_cast<const __half*>(L.gamma);
  g.wscale = reinterpret_cast<const __half*>(L.wscale);
  g.ascale = reinterpret_cast<const __half*>(L.ascale);
  g.rope = L.rope;
  g.ctl = make_ctl();
  if (g.num_tiles == 0) return QVGGT_OK;

  auto kfn = gemm_kernel<BN, MODE>;
  static DeviceFlags attr_set;
  if ((rc = ensure_smem(attr_set, kfn, C::SMEM, "cudaFuncSetAttribute(gemm)"))) return rc;
  const int grid = g.num_tiles < di.num_sms ? g.num_tiles : di.num_sms;
  return check_cuda(launch_pdl(kfn, dim3(grid), dim3(C::THREADS), C::SMEM, L.stream, 1u, tmA, tmB, tmS, tmZ, g),
                    "gemm launch");
}

}  // namespace

int gemm_launch(const GemmLaunch& L) {
  // Shape and layout checks shared by all modes.
  if (L.M < 0 || L.N <= 0 || L.K <= 0) return set_error(QVGGT_ERR_INVALID, "gemm: bad shape M=%lld N=%lld K=%lld",
                                                        (long long)L.M, (long long)L.N, (long long)L.K);
  if (L.N % 128 != 0) return set_error(QVGGT_ERR_UNSUPPORTED, "gemm: N=%lld must be a multiple of 128", (long long)L.N);
  const int kmul = (L.mode == B_I8) ? 128 : 64;
  if (L.K % kmul != 0)
    return set_error(QVGGT_ERR_UNSUPPORTED, "gemm: K=%lld must be a multiple of %d", (long long)L.K, kmul);
  if (!aligned16(L.a) || !aligned16(L.b) || !aligned16(L.out) || (L.bias && !aligned16(L.bias)))
    return set_error(QVGGT_ERR_ALIGN, "gemm: operands must be 16-byte aligned");
  if (L.mode < B_W4 || L.mode > B_W4BF) return set_error(QVGGT_ERR_INVALID, "gemm: mode %d", L.mode);
  if (L.mode == B_W4BF && L.epi != EPI_STORE)
    return set_error(QVGGT_ERR_UNSUPPORTED, "gemm: bf16 activations take the plain store epilogue only");
  if (mode_is_w4(L.mode)) {
    if (L.group_size <= 0 || L.group_size % 64 != 0 || L.K % L.group_size != 0)
      return set_error(QVGGT_ERR_UNSUPPORTED, "gemm: group_size=%d must be a multiple of 64 dividing K=%lld",
                       L.group_size, (long long)L.K);
    if (L.gpad < L.K / L.group_size) return set_error(QVGGT_ERR_INVALID, "gemm: scale table has too few groups");
    if (!aligned16(L.scales) || !aligned16(L.zeros)) return set_error(QVGGT_ERR_ALIGN, "gemm: scales not aligned");
  }
  if (L.epi == EPI_RESID && (!L.resid || !L.gamma)) return set_error(QVGGT_ERR_INVALID, "gemm: residual needs resid+gamma");
  if (L.epi == EPI_QKV_ROPE) {
    const RopeEpi& R = L.rope;
    if (L.mode == B_I8 || R.dim <= 0 || R.dim % 64 || L.N != 3 * R.dim || !R.q_out || !R.kv_out || !R.cos_tab ||
        !R.sin_tab || R.max_pos <= 0 || R.tokens_per_frame <= 0 || R.grid_w <= 0 || R.patch_start < 0)
      return set_error(QVGGT_ERR_INVALID, "gemm: bad qkv/rope epilogue arguments");
    if ((R.qn_w != nullptr) != (R.kn_w != nullptr) || (R.qn_w && (!R.qn_b || !R.kn_b)))
      return set_error(QVGGT_ERR_INVALID, "gemm: qk-norm needs all four weight vectors");
    if (!aligned16(R.q_out) || !aligned16(R.kv_out) || !aligned16(R.cos_tab) || !aligned16(R.sin_tab))
      return set_error(QVGGT_ERR_ALIGN, "gemm: rope epilogue tensors must be 16-byte aligned");
  }
  if (L.mode == B_I8 && L.epi != EPI_I32 && (!L.wscale || !L.ascale)) return set_error(QVGGT_ERR_INVALID, "gemm: w8a8 needs scales");
  if (L.M == 0) return QVGGT_OK;

  int cfg = gemm_config_override();
  const bool can256 = (L.N % 256 == 0) && !L.force_bn128;
  const bool can_pair = can256 && L.M >= 512;
  if ((cfg == GEMM_CFG_PAIR && !can_pair) || (cfg == GEMM_CFG_1SM_256 && !can256)) cfg = GEMM_CFG_AUTO;
  if (cfg == GEMM_CFG_AUTO) cfg = choose_gemm_config(L.mode, L.M, L.N, device_info().num_sms, can_pair, can256);
  switch (cfg) {
    case GEMM_CFG_PAIR: return gemm_launch_2sm(L);
    case GEMM_CFG_1SM_256:
      switch (L.mode) {
        case B_W4: return launch_gemm<256, B_W4>(L);
        case B_W4BF: return launch_gemm<256, B_W4BF>(L);
        case B_F16: return launch_gemm<256, B_F16>(L);
        default: return launch_gemm<256, B_I8>(L);
      }
    default:
      switch (L.mode) {
        case B_W4: return launch_gemm<128, B_W4>(L);
        case B_W4BF: return launch_gemm<128, B_W4BF>(L);
        case B_F16: return launch_gemm<128, B_F16>(L);
        default: return launch_gemm<128, B_I8>(L);
      }
  }
}

// Tuning override of the kernel configuration (-1: not read from the
// environment yet).  Set by qvggt_set_gemm_config.
std::atomic<int> g_gemm_cfg{-1};

int gemm_config_override() {
  int c = g_gemm_cfg.load(std::memory_order_relaxed);
  if (c < 0) {
    // QVGGT_GEMM_CONFIG = 0 (auto), 1 (CTA pairs), 2 (1-SM, 256-wide), 3 (1-SM, 128-wide)
    const char* e = getenv("QVGGT_GEMM_CONFIG");
    c = (e && e[0] >= '0' && e[0] <= '3' && e[1] == 0) ? e[0] - '0' : GEMM_CFG_AUTO;
    g_gemm_cfg.store(c, std::memory_order_relaxed);
  }
  return c;
}

// Kernel configuration for an M x N GEMM: the one with the least estimated
// time = (waves of tiles over the SMs) x (time of one tile).  Throughput of
// each kernel with the SMs full, measured on B200 at M = 43,968 over the
// aggregator's four linears (`profile_cases.py gemm_configs`): dense fp16
// pairs 1110-1320, 1-SM 256-wide 1000-1190, 128-wide 730-850 TFLOP/s; W4A16
// pairs 910-1090, 1-SM 700-780 / 530-560; int8 (no pair form) 1216 TOPS on
// the 256-wide kernel.  A pair tile is 256 x 256 on two SMs, a 1-SM tile
// 128 x BN on one.  With these rates pairs win for fp16 and W4A16 at every
// row count of the frame-sharded runs (5,496 to 43,968 rows; measured the
// same way), int8 takes the 256-wide 1-SM kernel.
int choose_gemm_config(int mode, long long M, long long N, int sms, bool can_pair, bool can256) {
  static const double rate[3][3] = {// [mode][pair, 1sm256, 1sm128]
                                    {1000.0, 760.0, 540.0},
                                    {1250.0, 1100.0, 780.0},
                                    {0.0, 1216.0, 850.0}};
  const int m = mode == B_W4BF ? B_W4 : (mode < 0 || mode > 2 ? 1 : mode);
  double best = 1e300;
  int pick = GEMM_CFG_1SM_128;
  auto consider = [&](int cfg, long long tiles, int slots, double tile_flop, double r) {
    if (r <= 0.0 || slots <= 0) return;
    const double waves = (double)((tiles + slots - 1) / slots);
    const double t = waves * tile_flop / r;   // per-SM work of one tile over that SM's share of the rate
    if (t < best * 0.98) {
      best = t;
      pick = cfg;
    }
  };
  const long long m128 = (M + 127) / 128, m256 = (M + 255) / 256;
  consider(GEMM_CFG_1SM_128, m128 * (N / 128), sms, 128.0 * 128.0, rate[m][2]);
  if (can256) consider(GEMM_CFG_1SM_256, m128 * (N / 256), sms, 128.0 * 256.0, rate[m][1]);
  if (can_pair) consider(GEMM_CFG_PAIR, m256 * (N / 256), sms / 2, 128.0 * 256.0, rate[m][0]);
  return pick;
}

}  // namespace qv

extern "C" int qvggt_set_gemm_config(int32_t cfg) {
  if (cfg < qv::GEMM_CFG_AUTO || cfg > qv::GEMM_CFG_1SM_128)
    return qv::set_error(QVGGT_ERR_INVALID, "set_gemm_config: %d is not 0 (auto), 1 (pairs), 2 or 3 (1-SM)", cfg);
  qv::g_gemm_cfg.store(cfg, std::memory_order_relaxed);
  return QVGGT_OK;
}

