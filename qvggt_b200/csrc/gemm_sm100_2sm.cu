// 2-SM tcgen05 GEMM for sm_100a: the same three operand modes and fused
// epilogues as gemm_sm100.cu, computed by CTA pairs (clusters of 2).
//
// A pair owns a 256 x 256 output tile.  Each CTA loads only its own 128 rows
// of A and its own half (128 columns) of B per 128-byte k-block (W4: packs and
// dequantises only its own 128 output channels); one thread of the even CTA
// issues tcgen05.mma.cta_group::2 with M = 256, which reads the A rows and B
// halves from both CTAs' shared memory and leaves each CTA's 128 rows of the
// accumulator in its own TMEM.  Per SM this halves the B bytes pulled from L2
// (dense / int8 modes) or the dequantisation work (W4) for the same tensor
// work, while each SM still double-buffers its 2 x 256 accumulator columns.
//
// Signalling across the pair: TMA loads of both CTAs complete on the even
// CTA's `full` barrier; the MMA commits are multicast to both CTAs' `empty`
// and `tmem_full` barriers; epilogue warps of both CTAs arrive on the even
// CTA's `tmem_empty` barriers (mapa addresses).  W4: the packed weights,
// scales and zeros come through their own stage ring and producer warp
// (warp 2); the dequant warps release a stage (`empty_b`) after a proxy fence
// that retires their ordinary loads of it, since the next TMA refills it.
// Dequantisation buffer d
// of k-block j is free once the MMAs of k-block j - ND are done, which the
// dequant warps read from that k-block's `empty` barrier (no barrier or commit
// of its own).  Each dequant warp then signals the even CTA with a 16-byte
// DSMEM bulk copy (cp.async.bulk shared::cta -> shared::cluster) that
// completes its bytes on `full_d[d]`, armed by the MMA thread with expect_tx
// for all eight warps' copies; the even CTA's warps first wait for both CTAs'
// A tiles (`full`), so the MMA thread waits on `full_d` alone, at CTA scope
// like on a TMA-completed barrier.  (A cluster-scope acquire cost the MMA
// thread ~0.15 us per k-block, and a cluster-scope release arrive costs its
// thread close to a microsecond.)  Every wait is bounded; both CTAs meet in a
// cluster barrier before TMEM is freed and before either exits; a CTA that
// aborted also marks its peer and both pause before exit so that no bulk copy
// in flight outlives its source or destination.  No multicast loads.
#include "gemm_common.cuh"
#include "gemm_sm100.cuh"
#include "host.hpp"

namespace qv {
namespace {

using namespace gemmk;

constexpr int HM = 128;      // rows per CTA (the pair tile has 256)
constexpr int KBB = 128;     // bytes of K per k-block
constexpr int PBN = 256;     // columns of the pair tile; each CTA holds PBN/2 of B
constexpr int HBN = PBN / 2;

template <int MODE>
struct Cfg2 {
  static constexpr int NS = 6;
  static constexpr int ND = (mode_is_w4(MODE)) ? 4 : 0;
  static constexpr int A_BYTES = HM * KBB;                                  // 16 KB
  static constexpr int B_BYTES = HBN * KBB;                                 // 16 KB: this CTA's half
  static constexpr int BQ_BYTES = (mode_is_w4(MODE)) ? (HBN / 4) * KBB : 0;     // 4 KB packed int4
  static constexpr int SZ_BYTES = (mode_is_w4(MODE)) ? 2 * HBN * 2 : 0;         // scales + zeros
  // W4: two groups of HBN/32 dequantisation warps take alternate k-blocks, so
  // two k-blocks are dequantised at once (NS and ND are even).
  static constexpr int DQ_GROUP_WARPS = (mode_is_w4(MODE)) ? HBN / 32 : 0;
  static constexpr int NUM_DQ_WARPS = 2 * DQ_GROUP_WARPS;
  static constexpr int THREADS = 256 + NUM_DQ_WARPS * 32;
  static_assert(NS % 2 == 0 && (ND % 2 == 0), "dequant groups alternate stages");
  // barriers first, then the 1024-aligned operand stages, then a 16 KB guard
  // so that every operand read of the pair MMA stays inside this CTA's
  // allocation even for a full-width B tile.
  static constexpr int OFF_BAR = 0;
  static constexpr int NUM_BARS = 4 * NS + ND + 4 + 1;
  // W4: buffer d = j % ND is reused by k-block j once the MMAs of j - ND are
  // done, read from empty[(j - ND) % NS].  NS - ND even and positive: the next
  // phase of that barrier needs the MMAs of j - ND + NS, whose B the same
  // dequant group produces after k-block j, so the parity wait cannot alias.
  static_assert(!mode_is_w4(MODE) || (NS > ND && (NS - ND) % 2 == 0), "W4 buffer reuse needs NS - ND even, > 0");
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int OFF_A = 1024;
  static constexpr int OFF_B = OFF_A + NS * A_BYTES;                        // dense B stages / W4 packed stages
  static constexpr int OFF_D = OFF_B + NS * ((mode_is_w4(MODE)) ? BQ_BYTES : B_BYTES);
  static constexpr int OFF_SZ = OFF_D + ND * B_BYTES;
  static constexpr int END = OFF_SZ + NS * SZ_BYTES;
  static constexpr int SMEM = END + HBN * KBB + 1024;                       // + guard + alignment slack
  static constexpr int OFF_SIG = 768;                                       // 16 B bulk-copy slot per dequant warp
  static constexpr uint32_t SIG_BYTES = 16;
  static constexpr uint32_t SIG_TX = 2 * DQ_GROUP_WARPS * SIG_BYTES;        // both CTAs' copies per k-block
  static_assert(OFF_MISC + 16 <= OFF_SIG && OFF_SIG + 2 * NUM_DQ_WARPS * 16 <= OFF_A, "barrier region overflow");
  static constexpr uint32_t TMEM_COLS = 2 * PBN;                            // 512: two accumulators
};

template <int MODE>
__global__ void __launch_bounds__(Cfg2<MODE>::THREADS, 1)
    gemm2sm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmS, const __grid_constant__ CUtensorMap tmZ, GemmArgs g) {
  using C = Cfg2<MODE>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* full = bars;                   // [NS] both CTAs' TMA -> MMA (even CTA's copy is used)
  uint64_t* empty = bars + C::NS;          // [NS] MMA -> producers (multicast)
  uint64_t* full_b = bars + 2 * C::NS;     // [NS] local TMA -> local dequant (W4)
  uint64_t* empty_b = bars + 3 * C::NS;    // [NS] local dequant -> local producer (W4)
  uint64_t* full_d = bars + 4 * C::NS;     // [ND] both CTAs' dequant warps -> MMA (even CTA's copy)
  uint64_t* tmem_full = full_d + C::ND;    // [2] MMA -> epilogue (multicast)
  uint64_t* tmem_empty = tmem_full + 2;    // [2] both CTAs' epilogue -> MMA (even CTA's copy)
  uint64_t* drain_bar = tmem_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster = blockIdx.x / 2, num_clusters = gridDim.x / 2;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
      mbar_init(&full_b[i], 1);
      mbar_init(&empty_b[i], C::DQ_GROUP_WARPS > 0 ? C::DQ_GROUP_WARPS : 1);
    }
    for (int i = 0; i < C::ND; ++i) {
      mbar_init(&full_d[i], 1);                      // the MMA thread's expect_tx arrival
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tmem_full[i], 1);
      mbar_init(&tmem_empty[i], 8);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    // first phase of each full_d: both CTAs' signal copies
    if (leader)
      for (int i = 0; i < C::ND; ++i) mbar_arrive_expect_tx(&full_d[i], C::SIG_TX);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
    tmem_relinquish_pair();
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
  cluster_sync();   // both CTAs' barriers exist before any cross-CTA signal
  tc_fence_after();
  // no global memory touched so far: wait for the previous kernel in the
  // stream only now (programmatic dependent launch)
  pdl_wait();
  pdl_trigger();
  const uint32_t tmem_base = *tmem_slot;
  const int num_kb = g.num_kb;

  if (warp == 0 || (mode_is_w4(MODE) && warp == 2)) {
    // ------------------------------------------------------------ producers (both CTAs)
    // Warp 0 loads A (and, dense / int8, B) into the stage ring paced by the
    // MMAs (`empty`).  W4: warp 2 loads the packed weights, scales and zeros
    // on their own pace, released by the dequant warps as soon as they have
    // read them (`empty_b`), so the dequantisation of a k-block never waits
    // behind the A tile of an earlier one.
    if (lane == 0) {
      const bool b_role = mode_is_w4(MODE) && warp == 2;
      uint32_t it = 0;
      bool ok = true;
      for (int tile = cluster; tile < g.num_tiles && ok; tile += num_clusters) {
        const int m_blk = tile / g.n_blocks, n_blk = tile % g.n_blocks;
        const int row0 = m_blk * 2 * HM + (int)rank * HM;       // this CTA's A rows
        const int col0 = n_blk * PBN + (int)rank * HBN;         // this CTA's B columns (output channels)
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % C::NS;
          const uint32_t ph = (it / C::NS) & 1;
          if (b_role) {
            if (!mbar_wait(&empty_b[s], ph ^ 1, abort_flag, g.ctl, ST_TIMEOUT_TMA_EMPTY)) { ok = false; break; }
            uint8_t* sq = smem + C::OFF_B + s * C::BQ_BYTES;
            uint8_t* ssz = smem + C::OFF_SZ + s * C::SZ_BYTES;
            const int grp = (kb * 64) / g.group_size;
            mbar_arrive_expect_tx(&full_b[s], C::BQ_BYTES + C::SZ_BYTES);
            tma_load_2d(sq, &tmB, &full_b[s], kb * 64, col0 / 4);
            tma_load_2d(ssz, &tmS, &full_b[s], col0, grp);
            tma_load_2d(ssz + HBN * 2, &tmZ, &full_b[s], col0, grp);
            continue;
          }
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, g.ctl, ST_TIMEOUT_TMA_EMPTY)) { ok = false; break; }
          const uint32_t full_lead = mapa_shared(&full[s], 0);
          uint8_t* sa = smem + C::OFF_A + s * C::A_BYTES;
          const int kx = kb * KBB / (MODE == B_I8 ? 1 : 2);
          if constexpr (mode_is_w4(MODE)) {
            if (leader) mbar_arrive_expect_tx(&full[s], 2 * C::A_BYTES);
            tma_load_2d_pair(sa, &tmA, full_lead, kx, row0);
          } else {
            uint8_t* sb = smem + C::OFF_B + s * C::B_BYTES;
            if (leader) mbar_arrive_expect_tx(&full[s], 2 * (C::A_BYTES + C::B_BYTES));
            tma_load_2d_pair(sa, &tmA, full_lead, kx, row0);
            tma_load_2d_pair(sb, &tmB, full_lead, kx, col0);
          }
        }
      }
      if (!ok) {
        // Let loads already issued land before this CTA can exit: wait for the
        // stage barriers this CTA can observe (the A producer: the even CTA's
        // full barriers of the last phases -- the MMA side has aborted too;
        // the W4 weight producer: the local full_b barriers).
        const uint32_t issued = it;
        for (int s = 0; s < C::NS; ++s) {
          const uint32_t cnt = issued > (uint32_t)s ? (issued - 1 - s) / C::NS + 1 : 0;
          if (cnt == 0) continue;
          if (b_role) mbar_wait_drain(&full_b[s], (cnt - 1) & 1, 200000000ull);
          else if (leader) mbar_wait_drain(&full[s], (cnt - 1) & 1, 200000000ull);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    if (leader && lane == 0) {
      constexpr uint32_t idesc = (MODE == B_I8) ? idesc_i8(2 * HM, PBN) : idesc_f16(2 * HM, PBN, false, false, MODE == B_W4BF);
      // This single thread paces the tensor core, so its per-k-block path is
      // kept short: stage / phase / dequant-buffer indices advance
      // incrementally, and the shared-memory descriptors are built once per
      // buffer base and advanced by adding the encoded byte offset (the start
      // address field holds address >> 4 and cannot carry below 256 KB).
      const uint64_t a_desc0 = sdesc_sw128(smem_u32(smem + C::OFF_A));
      const uint64_t b_desc0 = sdesc_sw128(smem_u32(smem + ((mode_is_w4(MODE)) ? C::OFF_D : C::OFF_B)));
      int s = 0, d = 0;
      uint32_t ph = 0, dph = 0;
      int t_local = 0;
      bool ok = true;
      for (int tile = cluster; tile < g.num_tiles && ok; tile += num_clusters, ++t_local) {
        const int acc = t_local & 1;
        const uint32_t aph = (t_local >> 1) & 1;
        if (!mbar_wait_cluster(&tmem_empty[acc], aph ^ 1, abort_flag, g.ctl, ST_TIMEOUT_TMEM)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * PBN;
        for (int kb = 0; kb < num_kb; ++kb) {
          // `full` completes through both CTAs' TMA transactions (complete_tx,
          // no software arrivals): a CTA-scope wait suffices, and a
          // cluster-scope acquire costs ~0.2 us per k-block on B200.  In W4
          // mode the even CTA's dequant warps have waited on it before
          // signalling full_d.
          if (!mode_is_w4(MODE) && !mbar_wait(&full[s], ph, abort_flag, g.ctl, ST_TIMEOUT_FULL)) { ok = false; break; }
          uint64_t bd;
          if constexpr (mode_is_w4(MODE)) {
            // completes through both CTAs' signal copies (complete_tx):
            // CTA scope, like `full`; then arm the buffer's next phase (its
            // copies come only after the commit below frees the buffer)
            if (!mbar_wait(&full_d[d], dph, abort_flag, g.ctl, ST_TIMEOUT_DEQ)) { ok = false; break; }
            mbar_arrive_expect_tx(&full_d[d], C::SIG_TX);
            bd = b_desc0 + (uint64_t)((d * C::B_BYTES) >> 4);
          } else {
            bd = b_desc0 + (uint64_t)((s * C::B_BYTES) >> 4);
          }
          tc_fence_after();
          const uint64_t ad = a_desc0 + (uint64_t)((s * C::A_BYTES) >> 4);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            if constexpr (MODE == B_I8)
              mma_i8_ss_pair(d_tmem, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
            else
              mma_f16_ss_pair(d_tmem, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
          }
          tc_commit_pair(&empty[s], 3);
          if constexpr (mode_is_w4(MODE)) {
            if (++d == C::ND) { d = 0; dph ^= 1; }
          }
          if (++s == C::NS) { s = 0; ph ^= 1; }
        }
        if (!ok) break;
        tc_commit_pair(&tmem_full[acc], 3);
      }
      if (!ok) {
        tc_commit(drain_bar);
        mbar_wait_drain(drain_bar, 0, 200000000ull);
      }
    }
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp - 4;
    const uint32_t tmem_empty_lead0 = mapa_shared(&tmem_empty[0], 0);
    const uint32_t tmem_empty_lead1 = mapa_shared(&tmem_empty[1], 0);
    int t_local = 0;
    for (int tile = cluster; tile < g.num_tiles; tile += num_clusters, ++t_local) {
      const int m_blk = tile / g.n_blocks, n_blk = tile % g.n_blocks;
      const int acc = t_local & 1;
      const uint32_t aph = (t_local >> 1) & 1;
      if (!mbar_wait_warp(&tmem_full[acc], aph, abort_flag, g.ctl, ST_TIMEOUT_TMEM)) break;
      tc_fence_after();
      const int row = m_blk * 2 * HM + (int)rank * HM + q * 32 + lane;
      const uint32_t tbase = tmem_addr(tmem_base, q * 32, acc * PBN);
      if (MODE != B_I8 && MODE != B_W4BF && g.epi == EPI_QKV_ROPE) {
#pragma unroll 1
        for (int c = 0; c < PBN / 64; ++c) {
          uint32_t r[64];
          tmem_ld32(tbase + c * 64, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
          tmem_ld32(tbase + c * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
          tmem_ld_wait();
          if (row < g.M) epilogue_qkv_head(g, row, n_blk * PBN + c * 64, r);
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < PBN / 16; ++c) {
          uint32_t r[16];
          tmem_ld16(tbase + c * 16, r);
          tmem_ld_wait();
          if (row < g.M) epilogue16<MODE>(g, row, n_blk * PBN + c * 16, r);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc ? tmem_empty_lead1 : tmem_empty_lead0);
    }
  } else if (warp >= 8) {
    // ------------------------------------------------------------ dequantisation (both CTAs)
    if constexpr (mode_is_w4(MODE)) {
      const int dq = threadIdx.x - 256;
      const uint32_t group = (uint32_t)(dq / HBN);   // takes the k-blocks with it % 2 == group
      const int n = dq % HBN;           // local output channel, 0..HBN-1
      const int grow = n >> 2;
      const int ci = n & 3;
      const int slot = (int)rank * C::NUM_DQ_WARPS + (warp - 8);
      const uint32_t sig_src = smem_u32(smem + C::OFF_SIG + slot * 16);
      const uint32_t sig_dst = mapa_shared(smem + C::OFF_SIG + slot * 16, 0);
      uint32_t it = 0;
      for (int tile = cluster; tile < g.num_tiles; tile += num_clusters) {
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          if ((it & 1u) != group) continue;
          const int s = it % C::NS;
          const uint32_t ph = (it / C::NS) & 1;
          if (!mbar_wait_warp(&full_b[s], ph, abort_flag, g.ctl, ST_TIMEOUT_FULL)) { ok = false; break; }
          const uint8_t* sq = smem + C::OFF_B + s * C::BQ_BYTES + grow * 128;
          const uint16_t* ssz = reinterpret_cast<const uint16_t*>(smem + C::OFF_SZ + s * C::SZ_BYTES);
          uint32_t x0[4], x1[4];
          *reinterpret_cast<uint4*>(x0) = *reinterpret_cast<const uint4*>(sq + (((2 * ci) ^ (grow & 7)) * 16));
          *reinterpret_cast<uint4*>(x1) = *reinterpret_cast<const uint4*>(sq + (((2 * ci + 1) ^ (grow & 7)) * 16));
          const uint32_t s2 = dup16(ssz + n);
          const uint32_t z2 = dup16(ssz + HBN + n);
          // the stage is refilled by TMA once released: retire these reads first
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty_b[s]);
          const int d = it % C::ND;
          // buffer d is free once the MMAs of k-block it - ND are done
          if (it >= (uint32_t)C::ND) {
            const uint32_t jf = it - C::ND;
            if (!mbar_wait_warp(&empty[jf % C::NS], (jf / C::NS) & 1, abort_flag, g.ctl, ST_TIMEOUT_DEQ)) {
              ok = false;
              break;
            }
          }
          uint8_t* drow = smem + C::OFF_D + d * C::B_BYTES + n * 128;
          uint4 o[4];
          dequant_chunk<MODE == B_W4BF>(x0, s2, z2, o);
#pragma unroll
          for (int qq = 0; qq < 4; ++qq) *reinterpret_cast<uint4*>(drow + ((qq ^ (n & 7)) * 16)) = o[qq];
          dequant_chunk<MODE == B_W4BF>(x1, s2, z2, o);
#pragma unroll
          for (int qq = 0; qq < 4; ++qq) *reinterpret_cast<uint4*>(drow + (((4 + qq) ^ (n & 7)) * 16)) = o[qq];
          fence_proxy_async_smem();
          // the even CTA's warps also take the wait for both CTAs' A tiles
          // off the MMA thread
          if (leader && !mbar_wait_warp(&full[s], ph, abort_flag, g.ctl, ST_TIMEOUT_FULL)) { ok = false; break; }
          __syncwarp();
          if (lane == 0) bulk_copy_to_cluster(sig_dst, sig_src, C::SIG_BYTES, mapa_shared(&full_d[d], 0));
        }
        if (!ok) break;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  // An abort in either CTA marks both, so both see it after the cluster barrier.
  if (threadIdx.x == 0 && *abort_flag) st_cluster_u32(mapa_shared(const_cast<int*>(abort_flag), rank ^ 1u), 1u);
  cluster_sync();   // neither CTA frees TMEM or exits while its peer may still use the pair
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
  if constexpr (mode_is_w4(MODE)) {
    // After an abort, W4 signal copies issued before the cluster barrier may
    // still be in flight: let them land before either CTA exits.
    if (*abort_flag) {
      const uint64_t t0 = globaltimer_ns();
      while (globaltimer_ns() - t0 < 50000ull) {
      }
    }
  }
}

template <int MODE>
int launch2(const GemmLaunch& L) {
  using C = Cfg2<MODE>;
  const DeviceInfo& di = device_info();
  if (C::SMEM > di.max_smem_optin)
    return set_error(QVGGT_ERR_UNSUPPORTED, "gemm2sm: %d B shared memory exceeds %d", C::SMEM, di.max_smem_optin);
  CUtensorMap tmA, tmB, tmS, tmZ;
  int rc;
  constexpr CUtensorMapDataType act_type =
      MODE == B_W4BF ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  if constexpr (MODE == B_I8) {
    rc = tmap_2d(&tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, L.a, L.K, L.M, L.lda, 128, HM, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = tmap_2d(&tmB, CU_TENSOR_MAP_DATA_TYPE_UINT8, L.b, L.K, L.N, L.K, 128, HBN, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    tmS = tmB;
    tmZ = tmB;
  } else {
    rc = tmap_2d(&tmA, act_type, L.a, L.K, L.M, L.lda * 2, 64, HM, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    if constexpr (mode_is_w4(MODE)) {
      rc = tmap_2d(&tmB, CU_TENSOR_MAP_DATA_TYPE_UINT16, L.b, L.K, L.N / 4, L.K * 2, 64, HBN / 4,
                   CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc) return rc;
      rc = tmap_2d(&tmS, act_type, L.scales, L.N, L.gpad, L.N * 2, HBN, 1,
                   CU_TENSOR_MAP_SWIZZLE_NONE);
      if (rc) return rc;
      rc = tmap_2d(&tmZ, act_type, L.zeros, L.N, L.gpad, L.N * 2, HBN, 1,
                   CU_TENSOR_MAP_SWIZZLE_NONE);
      if (rc) return rc;
    } else {
      rc = tmap_2d(&tmB, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, L.b, L.K, L.N, L.K * 2, 64, HBN, CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc) return rc;
      tmS = tmB;
      tmZ = tmB;
    }
  }
  GemmArgs g;
  g.M = (int)L.M;
  g.N = (int)L.N;
  g.K = (int)L.K;
  g.n_blocks = (int)(L.N / PBN);
  const int m_blocks = (int)((L.M + 2 * HM - 1) / (2 * HM));
  g.num_tiles = m_blocks * g.n_blocks;
  g.num_kb = (int)(L.K * (MODE == B_I8 ? 1 : 2) / KBB);
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

  auto kfn = gemm2sm_kernel<MODE>;
  static DeviceFlags attr_set;
  if ((rc = ensure_smem(attr_set, kfn, C::SMEM, "cudaFuncSetAttribute(gemm2sm)"))) return rc;
  const int max_clusters = di.num_sms / 2;
  const int clusters = g.num_tiles < max_clusters ? g.num_tiles : max_clusters;
  rc = check_cuda(launch_pdl(kfn, dim3(2 * clusters), dim3(C::THREADS), C::SMEM, L.stream, 2u, tmA, tmB, tmS, tmZ, g),
                  "gemm2sm launch");
  if (rc) return rc;
  return check_cuda(cudaGetLastError(), "gemm2sm launch");
}

}  // namespace

// Launches the 2-SM kernel for a shape gemm_launch has already validated;
// requires N % 256 == 0.
int gemm_launch_2sm(const GemmLaunch& L) {
  switch (L.mode) {
    case B_W4: return launch2<B_W4>(L);
    case B_W4BF: return launch2<B_W4BF>(L);
    case B_F16: return launch2<B_F16>(L);
    case B_I8: return launch2<B_I8>(L);
  }
  return set_error(QVGGT_ERR_INVALID, "gemm2sm: bad mode");
}

}  // namespace qv
