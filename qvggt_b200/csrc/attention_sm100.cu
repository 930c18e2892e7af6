// Flash attention, head_dim 64, non-causal, for sm_100a (tcgen05 + TMEM + TMA).
//
// One CTA per (batch, head, block of 256 query rows) = two 128-row Q tiles
// that share every K/V tile loaded into shared memory.  Per KV tile j of 128
// keys and Q tile i:
//   S_i = Q_i K_j^T        (tcgen05.mma, fp16 x fp16 -> fp32 in TMEM)
//   P_i = exp2(S_i*c - m)  (softmax warpgroup i: one thread per query row reads
//                           its whole S row from TMEM once, then computes)
//   O_i += P_i V_j         (tcgen05.mma with A = P read from TMEM, B = V from
//                           shared memory in the MN-major 128-byte-swizzled layout)
// Schedule: a softmax warpgroup releases S_i (s_free) as soon as its TMEM read
// of the row completes, so the tensor core computes S_i(j+1) while the
// warpgroup is still exponentiating tile j; P_i is written only after
// PV_i(j-1) has finished reading the previous P_i (o_done).  K and V stages
// are released separately: a K stage as soon as both S MMAs that read it
// complete, a V stage after both PV MMAs, and K and V have their own producer
// threads, so the K tiles for S(j+1..j+3) stream in while PV(j) still waits
// for the softmax of tile j.
// The running maximum m is only raised when a row's new maximum exceeds it by
// more than 2^8 (then O_i and the row sum are rescaled in place); P <= 256 fits
// fp16 and the final O / l is exact either way.
//
// Keys of a batch come from up to two row segments of the K/V buffer (a rank
// of a frame-sharded global block attends first to its own rows, then to the
// rows before and after them once the all-gather has landed), walked as one
// sequence of 128-key tiles; a tile that ends past its segment is masked.
// Split-KV: a (batch, head, query block) item may be cut into `splits` CTAs
// over consecutive ranges of that tile sequence (the grid then fills the
// 148 SMs in whole waves when the query blocks alone would leave a partial
// wave).  Each such CTA writes its normalised rows and their log-sum-exp to
// scratch, and the last of them to finish (a device-scope counter; no CTA
// ever waits for another) merges all of them.  lse_mode 1 also writes the
// log-sum-exp of every row; lse_mode 2 merges the result with an earlier call's
// (O in `out`, log-sum-exp in `lse`) over disjoint keys.
//
// TMEM columns: S0 [0,128) S1 [128,256) P0 [256,320) P1 [320,384)
//               O0 [384,448) O1 [448,512).
// Warps: 0 TMA producer of Q and K, 2 TMA producer of V, 1 TMEM owner + S
// MMA issuer, 3 PV MMA issuer, 4..7 softmax WG 0, 8..11 softmax WG 1.  All waits are bounded
// (common.cuh).
#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "host.hpp"

namespace qv {
namespace {

constexpr int KV_STAGES = 3;
constexpr int MAX_SPLITS = 4;          // KV splits per (batch, head, query block)
constexpr int TILE_BYTES = 128 * 128;  // 128 rows x 64 fp16
constexpr int THREADS = 384;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t COL_S0 = 0, COL_P0 = 256, COL_O0 = 384;

struct AttnSmem {
  // offsets from a 1024-aligned base
  static constexpr int Q0 = 0;
  static constexpr int Q1 = Q0 + TILE_BYTES;
  static constexpr int K = Q1 + TILE_BYTES;
  static constexpr int V = K + KV_STAGES * TILE_BYTES;
  static constexpr int BAR = V + KV_STAGES * TILE_BYTES;
  // barriers: q_full, k_full[S], v_full[S], k_empty[S], v_empty[S], s_full[2], s_free[2], p_full[2],
  // o_done[2], drain (S issuer), drain2 (PV issuer)
  static constexpr int NUM_BARS = 1 + 4 * KV_STAGES + 8 + 2 + 1;
  static constexpr int MISC = BAR + NUM_BARS * 8;
  // MISC: +0 TMEM base, +4 abort flag, +8 status word pointer, +16 timeout (ns),
  // +24 "this CTA merges the splits" flag, +28 first key tile of this CTA,
  // +32 + 4w the item softmax warp w (0..7) is on
  static constexpr int TOTAL = MISC + 64 + 1024;
};

struct AttnArgs {
  int batches, heads, nqb;
  int splits;                      // CTAs per (batch, head, query block)
  int nt0, nt;                     // 128-key tiles in segment 0, in both segments
  int seg0_start, seg0_len;        // key rows within a batch
  int seg1_start, seg1_len;        // (seg1_len 0: one segment)
  int lse_mode;                    // 0 none, 1 write lse, 2 merge with (out, lse) of an earlier call, write lse
  long long Lq, Lkv;
  __half* out;
  long long o_stride;
  float* lse;                      // [batches][heads][Lq], natural log of sum_k exp(q.k * scale)
  float* part_o;                   // [splits][batches * Lq][heads * 64]   (splits > 1)
  float* part_lse;                 // [splits][batches][heads][Lq]         (splits > 1)
  uint32_t* counters;              // [batches * heads * nqb], zero at launch (splits > 1)
  float scale_log2;
  Ctl ctl;
};

// First key row (within the batch) and number of valid keys of tile t of the
// two-segment key sequence.
__device__ __forceinline__ int tile_row(const AttnArgs& a, int t) {
  return t < a.nt0 ? a.seg0_start + t * 128 : a.seg1_start + (t - a.nt0) * 128;
}
__device__ __forceinline__ int tile_valid(const AttnArgs& a, int t) {
  const int rem = t < a.nt0 ? a.seg0_len - t * 128 : a.seg1_len - (t - a.nt0) * 128;
  return rem < 128 ? rem : 128;
}
// Tile range [t0, t1) of split `sp`.
__device__ __forceinline__ void split_range(const AttnArgs& a, int sp, int& t0, int& t1) {
  t0 = (int)((long long)sp * a.nt / a.splits);
  t1 = (int)((long long)(sp + 1) * a.nt / a.splits);
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Bounded mbarrier wait.  Its failure bookkeeping (abort flag, status word
// pointer, timeout) is read from shared memory at `misc` only once the first
// try_wait fails, so a thread keeps no registers for it across its loop (held
// in registers, it pushed parts of a softmax thread's 128-score row to local
// memory).
__device__ __forceinline__ bool wait_slow(uint32_t bar, uint32_t parity, uint32_t misc, uint32_t code) {
  int ab;
  uint64_t status, timeout;
  asm volatile("ld.shared.u64 %0, [%1 + 8];" : "=l"(status) : "r"(misc));
  asm volatile("ld.shared.u64 %0, [%1 + 16];" : "=l"(timeout) : "r"(misc));
  const uint64_t t0 = globaltimer_ns();
#pragma unroll 1
  while (true) {
    asm volatile("ld.volatile.shared.s32 %0, [%1 + 4];" : "=r"(ab) : "r"(misc) : "memory");
    if (ab) return false;
#pragma unroll 1
    for (int k = 0; k < 16; ++k)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > timeout) {
      asm volatile("st.volatile.shared.s32 [%0 + 4], 1;" ::"r"(misc) : "memory");
      if (status) atomicCAS(reinterpret_cast<uint32_t*>(status), 0u, code);
      return false;
    }
  }
}

__device__ __forceinline__ bool wait(uint32_t bar, uint32_t parity, uint32_t misc, uint32_t code) {
  return mbar_try_wait(bar, parity) || wait_slow(bar, parity, misc, code);
}
__device__ __forceinline__ bool wait(const uint64_t* bar, uint32_t parity, uint32_t misc, uint32_t code) {
  return wait(smem_u32(bar), parity, misc, code);
}

// The softmax warps' wait (barrier given by its shared-memory address): all
// lanes wait; the warp proceeds only if all saw the phase complete.
__device__ __forceinline__ bool softmax_wait(uint32_t bar, uint32_t parity, uint32_t misc) {
  return __all_sync(0xffffffffu, wait(bar, parity, misc, ST_TIMEOUT_SOFTMAX));
}

__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// Named barrier `id` over `count` threads (whole warps).
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ void arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// tcgen05.ld writes its destination registers asynchronously: they are valid
// only after tcgen05.wait::ld.  This empty asm takes s[A..B) as in-out
// operands after the wait, so the compiler cannot move reads of them above it.
template <int A, int B>
__device__ __forceinline__ void reg_fence(uint32_t (&s)[128]) {
#pragma unroll
  for (int k = A; k < B; ++k) asm volatile("" : "+r"(s[k]));
}

// Loads the thread's 128 S values (4 x 32 columns) with one wait.
__device__ __forceinline__ void load_s_row(uint32_t tS, uint32_t (&s)[128]) {
  tmem_ld32(tS + 0, *reinterpret_cast<uint32_t(*)[32]>(&s[0]));
  tmem_ld32(tS + 32, *reinterpret_cast<uint32_t(*)[32]>(&s[32]));
  tmem_ld32(tS + 64, *reinterpret_cast<uint32_t(*)[32]>(&s[64]));
  tmem_ld32(tS + 96, *reinterpret_cast<uint32_t(*)[32]>(&s[96]));
  tmem_ld_wait();
  reg_fence<0, 128>(s);
}

template <bool PARTIAL>
__device__ __forceinline__ float row_max(const uint32_t (&s)[128], int valid) {
  float m0 = -INFINITY, m1 = -INFINITY, m2 = -INFINITY, m3 = -INFINITY;
  if (!PARTIAL) {
    // three-input max: 64 instructions for 128 scores, four independent chains
#pragma unroll
    for (int e = 0; e < 128; e += 8) {
      m0 = max3f(m0, __uint_as_float(s[e + 0]), __uint_as_float(s[e + 1]));
      m1 = max3f(m1, __uint_as_float(s[e + 2]), __uint_as_float(s[e + 3]));
      m2 = max3f(m2, __uint_as_float(s[e + 4]), __uint_as_float(s[e + 5]));
      m3 = max3f(m3, __uint_as_float(s[e + 6]), __uint_as_float(s[e + 7]));
    }
  } else {
#pragma unroll
    for (int e = 0; e < 128; e += 4) {
      if (e + 0 < valid) m0 = fmaxf(m0, __uint_as_float(s[e + 0]));
      if (e + 1 < valid) m1 = fmaxf(m1, __uint_as_float(s[e + 1]));
      if (e + 2 < valid) m2 = fmaxf(m2, __uint_as_float(s[e + 2]));
      if (e + 3 < valid) m3 = fmaxf(m3, __uint_as_float(s[e + 3]));
    }
  }
  return fmaxf(fmaxf(m0, m1), fmaxf(m2, m3));
}

// 2^x for a pair of arguments on the FMA pipe (Cody-Waite range reduction:
// x = n + f, n = round(x), f in [-1/2, 1/2]; 2^f by a degree-3 polynomial
// fitted to minimise the relative error on [-1/2, 1/2] (max 7.5e-5, well under
// the fp16 rounding P gets afterwards); 2^n added into the exponent field).
// Arguments are clamped at -125 so 2^n stays a normal float; those values
// round to 0 in fp16 anyway.
__device__ __forceinline__ void exp2_poly_pair(uint64_t x2, float& p0, float& p1) {
  const uint64_t MAGIC = f2_pack(12582912.0f, 12582912.0f);        // 1.5 * 2^23: rounds to an integer
  const uint64_t NEG_MAGIC = f2_pack(-12582912.0f, -12582912.0f);
  const uint64_t NEG_ONE = f2_pack(-1.0f, -1.0f);
  const uint64_t C0 = f2_pack(0.99992806f, 0.99992806f), C1 = f2_pack(0.69326097f, 0.69326097f);
  const uint64_t C2 = f2_pack(0.24261114f, 0.24261114f), C3 = f2_pack(0.05517166f, 0.05517166f);
  float x0, x1;
  f2_unpack(x2, x0, x1);
  const uint64_t xc = f2_pack(fmaxf(x0, -125.f), fmaxf(x1, -125.f));
  const uint64_t t = f2_add(xc, MAGIC);          // low mantissa bits hold n
  const uint64_t nf = f2_add(t, NEG_MAGIC);      // n as a float
  const uint64_t f = f2_fma(nf, NEG_ONE, xc);    // x - n
  uint64_t p = f2_fma(C3, f, C2);
  p = f2_fma(p, f, C1);
  p = f2_fma(p, f, C0);
  float q0, q1, t0, t1;
  f2_unpack(p, q0, q1);
  f2_unpack(t, t0, t1);
  p0 = __int_as_float(__float_as_int(q0) + (__float_as_int(t0) << 23));
  p1 = __int_as_float(__float_as_int(q1) + (__float_as_int(t1) << 23));
}

// Pairs E0..E0+15 of p = exp2(s*c - m) (0 beyond `valid`), added into l2 and
// packed as fp16 pairs into s[E0..E0+15] (in place: chunk E0/16 reads scores
// s[2*E0..2*E0+31], which no earlier chunk wrote).  POLY of every 8 pairs use
// the FMA-pipe polynomial, the rest MUFU ex2 (16 results per SM per clock).
template <bool PARTIAL, int POLY, int E0>
__device__ __forceinline__ void exp_chunk(uint32_t (&s)[128], uint64_t c2, uint64_t nm2, uint64_t& l2, int valid) {
  // two partial sums (even / odd pairs) keep the add chain short
  uint64_t la = f2_pack(0.f, 0.f), lb = f2_pack(0.f, 0.f);
#pragma unroll
  for (int e = E0; e < E0 + 16; ++e) {
    const uint64_t x2 = f2_fma(f2_pack(__uint_as_float(s[2 * e]), __uint_as_float(s[2 * e + 1])), c2, nm2);
    float p0, p1;
    if ((e & 7) < POLY) {
      exp2_poly_pair(x2, p0, p1);
    } else {
      float x0, x1;
      f2_unpack(x2, x0, x1);
      p0 = ex2(x0);
      p1 = ex2(x1);
    }
    if (PARTIAL) {
      if (2 * e >= valid) p0 = 0.f;
      if (2 * e + 1 >= valid) p1 = 0.f;
    }
    if (e & 1) lb = f2_add(lb, f2_pack(p0, p1));
    else la = f2_add(la, f2_pack(p0, p1));
    s[e] = pack_half2(p0, p1);
  }
  l2 = f2_add(l2, f2_add(la, lb));
}

// P = exp2(S*c - m) for the thread's row, written to TMEM in four 16-column
// chunks as they are produced: each tcgen05.st is asynchronous until the one
// wait at the end, so three of the four stores overlap the exponentials still
// to come.  P may be written only once PV(j-1) has read the previous P: that
// wait (`o_ready` false) comes just before the first store.  Returns the row
// sum of P, or NaN if the wait gave up.
template <bool PARTIAL, int POLY>
__device__ __forceinline__ float exp_store(uint32_t (&s)[128], float c, float neg_m, int valid, uint32_t tP,
                                           bool o_ready, uint32_t o_done, uint32_t o_parity,
                                           uint32_t misc) {
  const uint64_t c2 = f2_pack(c, c), nm2 = f2_pack(neg_m, neg_m);
  uint64_t l2 = f2_pack(0.f, 0.f);
  exp_chunk<PARTIAL, POLY, 0>(s, c2, nm2, l2, valid);
  if (!o_ready) {
    if (!softmax_wait(o_done, o_parity, misc)) return __int_as_float(0x7fc00000);
    tc_fence_after();
  }
  tmem_st16(tP + 0, *reinterpret_cast<const uint32_t(*)[16]>(&s[0]));
  exp_chunk<PARTIAL, POLY, 16>(s, c2, nm2, l2, valid);
  tmem_st16(tP + 16, *reinterpret_cast<const uint32_t(*)[16]>(&s[16]));
  exp_chunk<PARTIAL, POLY, 32>(s, c2, nm2, l2, valid);
  tmem_st16(tP + 32, *reinterpret_cast<const uint32_t(*)[16]>(&s[32]));
  exp_chunk<PARTIAL, POLY, 48>(s, c2, nm2, l2, valid);
  tmem_st16(tP + 48, *reinterpret_cast<const uint32_t(*)[16]>(&s[48]));
  tmem_st_wait();
  float l0, l1;
  f2_unpack(l2, l0, l1);
  return l0 + l1;
}

// GENERAL = false: one split, no log-sum-exp (every single-GPU launch); its
// epilogue only normalises and stores O.  GENERAL = true adds the split
// merge and the log-sum-exp modes (their epilogue costs registers the plain
// launch should not pay for).
template <int POLY, bool GENERAL>
__global__ void __launch_bounds__(THREADS, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + AttnSmem::BAR);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + KV_STAGES;
  uint64_t* k_empty = v_full + KV_STAGES;   // [S] MMA -> K producer: S_0, S_1 of the tile done
  uint64_t* v_empty = k_empty + KV_STAGES;  // [S] MMA -> V producer: PV_0, PV_1 of the tile done
  // the four [2] arrays below are consecutive: the softmax warps address them
  // from s_full[i] at byte offsets 16, 32 and 48
  uint64_t* s_full = v_empty + KV_STAGES;   // [2] MMA -> softmax: S_i ready
  uint64_t* s_free = s_full + 2;            // [2] softmax -> MMA: S_i read
  uint64_t* p_full = s_free + 2;            // [2] softmax -> MMA: P_i written
  uint64_t* o_done = p_full + 2;            // [2] MMA -> softmax: PV_i complete
  uint64_t* drain = o_done + 2;
  uint64_t* drain2 = drain + 1;
  uint64_t* q_empty = drain2 + 1;           // S issuer -> Q producer: the item's S MMAs done with Q
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + AttnSmem::MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + AttnSmem::MISC + 4);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int sp = blockIdx.x % a.splits;          // KV split of this CTA
  // Work items are (batch, head, query block).  The plain kernel is
  // persistent: CTA x takes items x, x + gridDim.x, ... one after another,
  // every role walking the same sequence, so the next item's Q and first
  // K / V tiles load and its first S MMAs run while the current item's last
  // tiles and epilogue finish.  The general kernel takes one item per CTA.
  const int n_items = a.batches * a.heads * a.nqb;
  const int item0 = blockIdx.x / a.splits;
  const int item_step = GENERAL ? n_items : (int)gridDim.x;
  int t_first, t_end;
  split_range(a, sp, t_first, t_end);
  const int nkv = t_end - t_first;               // KV tiles of this CTA, per item

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < KV_STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_done[i], 1);
    }
    mbar_init(drain, 1);
    mbar_init(drain2, 1);
    mbar_init(q_empty, 1);
    *abort_flag = 0;
    *reinterpret_cast<uint32_t**>(smem + AttnSmem::MISC + 8) = a.ctl.status;
    *reinterpret_cast<unsigned long long*>(smem + AttnSmem::MISC + 16) = a.ctl.timeout_ns;
    *reinterpret_cast<int*>(smem + AttnSmem::MISC + 28) = t_first;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // the prologue above touches no global memory: wait for the previous
  // kernel in the stream only now (programmatic dependent launch)
  pdl_wait();
  pdl_trigger();
  const uint32_t tmem = *tmem_slot;
  const uint32_t misc = smem_u32(smem + AttnSmem::MISC);

  // Registers: launched at 168 per thread (384 x 168 = 64512); warpgroup 0
  // (producers, MMA issuers, which walk the two-segment tile sequence) gives
  // back to 64, the two softmax warpgroups take 216 each:
  // 128*64 + 256*216 = 63488 <= 64512.
  // setmaxnreg is warpgroup-collective: all four warps of a warpgroup must
  // execute the same one (a warpgroup whose warps disagree never completes
  // it, and the other warpgroups' increments then wait forever).
  if (warp < 4) {
    regs_dec<64>();
    if (warp == 0 || warp == 2) {
    // ------------------------------------------------------------ TMA producers (K + Q / V)
    if (lane == 0) {
      const bool is_k = warp == 0;
      const CUtensorMap* tm = is_k ? &tmK : &tmV;
      uint64_t* full = is_k ? k_full : v_full;
      uint64_t* empty = is_k ? k_empty : v_empty;
      uint8_t* base = smem + (is_k ? AttnSmem::K : AttnSmem::V);
      int jg = 0, it = 0;   // ring slots used, items started
      bool ok = true;
      for (int item = item0; ok && item < n_items; item += item_step, ++it) {
        const int qb = item % a.nqb;
        const int h = (item / a.nqb) % a.heads;
        const long long b = item / (a.nqb * a.heads);
        if (is_k) {
          // Q of the previous item is free once its S MMAs are done
          if (it > 0 && !wait(q_empty, (it - 1) & 1, misc, ST_TIMEOUT_TMA_EMPTY)) { ok = false; break; }
          const long long q_row0 = b * a.Lq + (long long)qb * 256;
          mbar_arrive_expect_tx(q_full, 2 * TILE_BYTES);
          tma_load_3d(smem + AttnSmem::Q0, &tmQ, q_full, 0, h, (int)q_row0);
          tma_load_3d(smem + AttnSmem::Q1, &tmQ, q_full, 0, h, (int)(q_row0 + 128));
        }
        const long long kv_row0 = b * a.Lkv;
        for (int j = 0; j < nkv; ++j, ++jg) {
          const int st = jg % KV_STAGES;
          const uint32_t ph = (jg / KV_STAGES) & 1;
          if (!wait(&empty[st], ph ^ 1, misc, ST_TIMEOUT_TMA_EMPTY)) { ok = false; break; }
          const int row = (int)(kv_row0 + tile_row(a, t_first + j));
          mbar_arrive_expect_tx(&full[st], TILE_BYTES);
          tma_load_3d(base + st * TILE_BYTES, tm, &full[st], 0, h, row);
        }
      }
      if (!ok) {
        // aborted: let the loads already issued land before the CTA exits
        if (is_k && it > 0) mbar_wait_drain(q_full, (it - 1) & 1, 200000000ull);
        for (int jj = (jg > KV_STAGES ? jg - KV_STAGES : 0); jj < jg; ++jj)
          mbar_wait_drain(&full[jj % KV_STAGES], (jj / KV_STAGES) & 1, 200000000ull);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ S = Q K^T issuer
    // S and PV MMAs are issued by two threads (warps 1 and 3): each
    // tcgen05.mma costs its issuing thread tens of cycles, so with one issuer
    // the next tile's S had to queue behind both PVs of the previous tile.
    // Each thread commits (and, on abort, drains) only its own MMAs.
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16(128, 128);
      const uint32_t q_addr[2] = {smem_u32(smem + AttnSmem::Q0), smem_u32(smem + AttnSmem::Q1)};
      uint32_t cs[2] = {0, 0};   // S_i tiles issued so far (across items)
      int jg = 0, it = 0;
      bool ok = true;
      for (int item = item0; ok && item < n_items; item += item_step, ++it) {
        // Q tiles of the item that hold rows of its batch (the last block of
        // a batch may end inside tile 0, e.g. 1374 = 5 x 256 + 94): an empty
        // tile 1 gets no MMAs and no softmax
        const int nqt = ((long long)(item % a.nqb) * 256 + 128 < a.Lq) ? 2 : 1;
        if (!wait(q_full, it & 1, misc, ST_TIMEOUT_FULL)) { ok = false; break; }
        for (int j = 0; j < nkv; ++j, ++jg) {
          const int st = jg % KV_STAGES;
          if (!wait(&k_full[st], (jg / KV_STAGES) & 1, misc, ST_TIMEOUT_FULL)) { ok = false; break; }
          const uint32_t k_addr = smem_u32(smem + AttnSmem::K + st * TILE_BYTES);
          for (int i = 0; i < nqt; ++i) {
            // S_i is free once softmax i has read the previous S_i
            if (cs[i] > 0 && !wait(&s_free[i], (cs[i] - 1) & 1, misc, ST_TIMEOUT_SOFTMAX)) {
              ok = false;
              break;
            }
            tc_fence_after();
#pragma unroll
            for (int k = 0; k < 4; ++k)
              mma_f16_ss(tmem + COL_S0 + i * 128, sdesc_sw128(q_addr[i] + k * 32), sdesc_sw128(k_addr + k * 32),
                         idesc_s, k > 0 ? 1u : 0u);
            tc_commit(&s_full[i]);
            ++cs[i];
          }
          if (!ok) break;
          tc_commit(&k_empty[st]);
        }
        if (ok) tc_commit(q_empty);   // the item's S MMAs are the last readers of its Q
      }
      if (!ok) {
        tc_commit(drain);
        mbar_wait_drain(drain, 0, 200000000ull);
      }
    }
  } else if (warp == 3) {
    // ------------------------------------------------------------ O += P V issuer
    if (lane == 0) {
      constexpr uint32_t idesc_o = idesc_f16(128, 64, false, true);   // B = V, MN-major
      uint32_t cp[2] = {0, 0};   // PV_i tiles issued so far (across items)
      int jg = 0;
      bool ok = true;
      for (int item = item0; ok && item < n_items; item += item_step) {
        const int nqt = ((long long)(item % a.nqb) * 256 + 128 < a.Lq) ? 2 : 1;
        for (int jj = 0; jj < nkv; ++jj, ++jg) {
          const int st = jg % KV_STAGES;
          const uint32_t v_addr = smem_u32(smem + AttnSmem::V + st * TILE_BYTES);
          for (int i = 0; i < nqt; ++i) {
            if (!wait(&p_full[i], cp[i] & 1, misc, ST_TIMEOUT_SOFTMAX)) { ok = false; break; }
            if (i == 0 && !wait(&v_full[st], (jg / KV_STAGES) & 1, misc, ST_TIMEOUT_FULL)) {
              ok = false;
              break;
            }
            tc_fence_after();
#pragma unroll
            for (int k = 0; k < 8; ++k)
              mma_f16_ts(tmem + COL_O0 + i * 64, tmem + COL_P0 + i * 64 + k * 8, sdesc_sw128(v_addr + k * 2048),
                         idesc_o, (jj > 0 || k > 0) ? 1u : 0u);
            tc_commit(&o_done[i]);
            ++cp[i];
          }
          if (!ok) break;
          tc_commit(&v_empty[st]);
        }
      }
      if (!ok) {
        tc_commit(drain2);
        mbar_wait_drain(drain2, 0, 200000000ull);
      }
    }
    }
  } else if (warp >= 4 && warp < 12) {
    // ------------------------------------------------------------ softmax WG i
    regs_inc<216>();
    const int i = (warp - 4) / 4;
    const int quarter = warp & 3;             // TMEM lane quarter
    const int r = quarter * 32 + lane;        // row within the Q tile
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + lane_base + COL_S0 + i * 128;
    const uint32_t tP = tmem + lane_base + COL_P0 + i * 64;
    const uint32_t tO = tmem + lane_base + COL_O0 + i * 64;
    const float c = a.scale_log2;
    const uint32_t bar_s_full = smem_u32(&s_full[i]);
    const uint32_t bar_s_free = bar_s_full + 16, bar_p_full = bar_s_full + 32, bar_o_done = bar_s_full + 48;
    uint32_t cnt = 0;   // S_i tiles taken so far (across items)
    bool ok = true;
    // the warp's current item lives in shared memory, not in a register held
    // through the tile loop (that pushed parts of the score row to local memory)
#define QV_ITEM_SLOT (misc + 32 + ((threadIdx.x >> 5) - 4) * 4)
    if (lane == 0) asm volatile("st.shared.s32 [%0], %1;" ::"r"(QV_ITEM_SLOT), "r"(item0) : "memory");
    __syncwarp();
    for (;;) {
    int item;
    asm volatile("ld.shared.s32 %0, [%1];" : "=r"(item) : "r"(QV_ITEM_SLOT) : "memory");
    if (!ok || item >= a.batches * a.heads * a.nqb) break;
    // a Q tile past the end of its batch has no MMAs; its warpgroup still
    // runs the epilogue (with nothing to store) so the split merge's named
    // barriers see both warpgroups
    const int nkv_i = i < (((long long)(item % a.nqb) * 256 + 128 < a.Lq) ? 2 : 1) ? nkv : 0;
    float m_used = -INFINITY, l = 0.f;
    for (int j = 0; ok && j < nkv_i; ++j, ++cnt) {
      if (!softmax_wait(bar_s_full, cnt & 1, misc)) { ok = false; break; }
      tc_fence_after();
      uint32_t s[128];
      load_s_row(tS, s);
      // S_i is in registers: hand the TMEM columns back to the MMA warp
      tc_fence_before();
      __syncwarp();
      if (lane == 0) arrive(bar_s_free);

      // the CTA's first tile is re-read from shared memory (a register
      // held through the loop pushed parts of the score row to local memory)
      int tf;
      asm volatile("ld.shared.s32 %0, [%1 + 28];" : "=r"(tf) : "r"(misc));
      const int valid = tile_valid(a, tf + j);
      const float mx = (valid == 128) ? row_max<false>(s, valid) : row_max<true>(s, valid);
      const float m_new = fmaxf(m_used, mx * c);
      const bool need = m_new > m_used + 8.0f;
      // Raising m rescales O_i and l by alpha; O_i is rescaled after the P
      // store, when PV_i(j-1) is known complete and the scores are no longer
      // held in registers.
      float alpha = 1.f;
      bool rescale = false;
      if (__any_sync(0xffffffffu, need)) {
        const float m_target = need ? m_new : m_used;
        alpha = (m_used == -INFINITY) ? 0.f : ex2(m_used - m_target);
        rescale = j > 0;
        m_used = m_target;
      }
      const uint32_t o_par = (cnt - 1) & 1;
      // PV_i(j-1) complete (nothing to wait for at j = 0: the previous item's
      // epilogue has waited for its last PV)
      const bool o_ready = j == 0;
      const float lj = (valid == 128)
          ? exp_store<false, POLY>(s, c, -m_used, valid, tP, o_ready, bar_o_done, o_par, misc)
          : exp_store<true, POLY>(s, c, -m_used, valid, tP, o_ready, bar_o_done, o_par, misc);
      if (__any_sync(0xffffffffu, lj != lj)) { ok = false; break; }
      l = l * alpha + lj;
      if (rescale) {
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          uint32_t v[16];
          tmem_ld16(tO + cc * 16, v);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 16; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * alpha);
          tmem_st16(tO + cc * 16, v);
        }
        tmem_st_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) arrive(bar_p_full);
    }
    // ------------------------------------------------------------ epilogue
    // `have`: O_i of the last tile is complete (warp-uniform, so the
    // warp-collective TMEM loads below run in whole warps).
    bool have = false;
    if (ok && nkv_i > 0) {
      have = softmax_wait(bar_o_done, (cnt - 1) & 1, misc);
      if (have) tc_fence_after();
    }
    // the split and the item are re-read here (%ctaid.x, shared memory)
    // rather than kept in registers through the loop
    uint32_t cta;
    asm volatile("mov.u32 %0, %%ctaid.x;" : "=r"(cta));
    const uint32_t sp_e = cta % (uint32_t)a.splits;
    uint32_t item_e;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(item_e) : "r"(QV_ITEM_SLOT) : "memory");
    const int qb_e = (int)(item_e % (uint32_t)a.nqb);
    const int h_e = (int)((item_e / (uint32_t)a.nqb) % (uint32_t)a.heads);
    const long long b_e = item_e / ((uint32_t)a.nqb * (uint32_t)a.heads);
    const long long qr = (long long)qb_e * 256 + i * 128 + r;   // row within the batch
    __half* dst = a.out + (b_e * a.Lq + qr) * a.o_stride + h_e * 64;
    if (!GENERAL) {
      if (have) {
        const float inv = 1.f / l;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          uint32_t v[16];
          tmem_ld16(tO + cc * 16, v);
          tmem_ld_wait();
          uint32_t o[8];
#pragma unroll
          for (int e = 0; e < 8; ++e)
            o[e] = pack_half2(__uint_as_float(v[2 * e]) * inv, __uint_as_float(v[2 * e + 1]) * inv);
          if (qr < a.Lq) {
            uint4* d4 = reinterpret_cast<uint4*>(dst + cc * 16);
            d4[0] = make_uint4(o[0], o[1], o[2], o[3]);
            d4[1] = make_uint4(o[4], o[5], o[6], o[7]);
          }
        }
      }
    } else {
      const bool row_ok = have && qr < a.Lq;
      // log2 of this CTA's sum over its keys of exp2(s * c) for the row
      const float lse2_own = m_used + log2f(l);
      const long long bhq = ((long long)b_e * a.heads + h_e) * a.Lq + qr;        // [b][h][row]
      const long long split_rows = (long long)a.batches * a.heads * a.Lq;       // rows of one split's parts
      bool merge = true;
      if (a.splits > 1) {
        // every split parks its normalised rows; the last to finish merges
        const long long part = (long long)sp_e * split_rows + bhq;
        if (have) {
          const float inv = 1.f / l;
          float4* po = reinterpret_cast<float4*>(a.part_o + part * 64);
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            uint32_t v[16];
            tmem_ld16(tO + cc * 16, v);
            tmem_ld_wait();
            if (row_ok) {
#pragma unroll
              for (int e = 0; e < 4; ++e)
                po[cc * 4 + e] = make_float4(__uint_as_float(v[4 * e]) * inv, __uint_as_float(v[4 * e + 1]) * inv,
                                             __uint_as_float(v[4 * e + 2]) * inv,
                                             __uint_as_float(v[4 * e + 3]) * inv);
            }
          }
          if (row_ok) a.part_lse[part] = lse2_own;
        }
        fence_acq_rel_gpu();
        named_bar_sync(1, 256);
        if (threadIdx.x == 4 * 32) {   // the first softmax thread counts the CTA in
          const uint32_t old = atom_add_acq_rel_gpu(a.counters + item_e, 1u);
          const uint32_t last = old == (uint32_t)a.splits - 1u;
          asm volatile("st.shared.u32 [%0 + 24], %1;" ::"r"(misc), "r"(last) : "memory");
        }
        named_bar_sync(1, 256);
        uint32_t last;
        asm volatile("ld.shared.u32 %0, [%1 + 24];" : "=r"(last) : "r"(misc) : "memory");
        merge = last != 0;
        if (merge) fence_acq_rel_gpu();
      }
      if (merge && have) {
        // Weights of every part of the row from their log2-sum-exps: with
        // splits, every split's parked part (this CTA's included, so the sum
        // runs in split order whichever CTA merges and results repeat bit for
        // bit); with one split, this CTA's O from TMEM; for lse_mode 2 the
        // earlier call's result last.  The row is merged 16 columns at a time.
        const bool own_tmem = a.splits == 1;
        float w_part[MAX_SPLITS];
        float lmax = own_tmem ? lse2_own : -INFINITY;
#pragma unroll
        for (int s2 = 0; s2 < MAX_SPLITS; ++s2) {
          w_part[s2] = -INFINITY;
          if (row_ok && !own_tmem && s2 < a.splits) {
            w_part[s2] = a.part_lse[(long long)s2 * split_rows + bhq];
            lmax = fmaxf(lmax, w_part[s2]);
          }
        }
        float w_prev = -INFINITY;
        if (row_ok && a.lse_mode == 2) {
          w_prev = a.lse[bhq] * 1.4426950408889634f;
          lmax = fmaxf(lmax, w_prev);
        }
        const float w_own = own_tmem ? ex2(lse2_own - lmax) : 0.f;
        float wsum = w_own;
#pragma unroll
        for (int s2 = 0; s2 < MAX_SPLITS; ++s2) {
          w_part[s2] = ex2(w_part[s2] - lmax);      // exp2(-inf) = 0 for absent parts
          wsum += w_part[s2];
        }
        w_prev = ex2(w_prev - lmax);
        wsum += w_prev;
        const float inv = 1.f / wsum;
        const float scale_own = w_own * inv / l;
#pragma unroll 1
        for (int cc = 0; cc < 4; ++cc) {
          float acc[16];
          if (own_tmem) {
            uint32_t v[16];
            tmem_ld16(tO + cc * 16, v);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 16; ++e) acc[e] = __uint_as_float(v[e]) * scale_own;
          } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) acc[e] = 0.f;
          }
          if (row_ok) {
#pragma unroll
            for (int s2 = 0; s2 < MAX_SPLITS; ++s2) {
              if (own_tmem || s2 >= a.splits) continue;
              const float w = w_part[s2] * inv;
              const float4* po = reinterpret_cast<const float4*>(a.part_o + ((long long)s2 * split_rows + bhq) * 64 +
                                                                 cc * 16);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float4 x = po[e];
                acc[4 * e] += w * x.x;
                acc[4 * e + 1] += w * x.y;
                acc[4 * e + 2] += w * x.z;
                acc[4 * e + 3] += w * x.w;
              }
            }
            if (a.lse_mode == 2) {
              const float w = w_prev * inv;
              const uint4* pv = reinterpret_cast<const uint4*>(dst + cc * 16);
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const uint4 u = pv[e];
                const uint32_t uu[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                  const float2 f = unpack_half2(uu[k]);
                  acc[8 * e + 2 * k] += w * f.x;
                  acc[8 * e + 2 * k + 1] += w * f.y;
                }
              }
            }
            uint4* d4 = reinterpret_cast<uint4*>(dst + cc * 16);
            d4[0] = make_uint4(pack_half2(acc[0], acc[1]), pack_half2(acc[2], acc[3]), pack_half2(acc[4], acc[5]),
                               pack_half2(acc[6], acc[7]));
            d4[1] = make_uint4(pack_half2(acc[8], acc[9]), pack_half2(acc[10], acc[11]),
                               pack_half2(acc[12], acc[13]), pack_half2(acc[14], acc[15]));
          }
        }
        if (row_ok && a.lse_mode != 0) a.lse[bhq] = (lmax + log2f(wsum)) * 0.6931471805599453f;
      }
    }
    __syncwarp();
    if (lane == 0)
      asm volatile("st.shared.s32 [%0], %1;" ::"r"(QV_ITEM_SLOT),
                   "r"((int)item_e + (GENERAL ? a.batches * a.heads * a.nqb : (int)gridDim.x))
                   : "memory");
    __syncwarp();
#undef QV_ITEM_SLOT
    }   // items
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace
}  // namespace qv

using namespace qv;

namespace qv {
namespace {

inline long long align256(long long x) { return (x + 255) & ~255LL; }

// Split count for `items` (batch, head, query block) items of `nt` key tiles
// each on `slots` concurrent CTAs (one per SM): the grid runs in
// ceil(items * s / slots) waves of CTAs that walk nt / s tiles plus a fixed
// cost (prologue, epilogue, split merge) of about two tiles; s is the
// cheapest of 1..MAX_SPLITS that keeps at least 8 tiles per split, taken only
// when it beats one split by more than 3 %.
int plan_splits(long long items, int nt, int slots) {
  if (slots <= 0 || items <= 0) return 1;
  auto cost = [&](int s) {
    const long long waves = (items * s + slots - 1) / slots;
    return (double)waves * ((double)nt / s + 2.0 * (s > 1 ? 1.5 : 1.0));
  };
  int best = 1;
  double best_cost = cost(1);
  for (int s = 2; s <= MAX_SPLITS && nt / s >= 8; ++s) {
    const double c = cost(s);
    if (c < best_cost * 0.97) {
      best = s;
      best_cost = c;
    }
  }
  return best;
}

struct ScratchLayout {
  long long counters, part_lse, part_o, total;   // byte offsets and size
};

ScratchLayout scratch_layout(long long batches, long long Lq, int heads, int splits) {
  ScratchLayout L{};
  if (splits <= 1) return L;
  const long long nqb = (Lq + 255) / 256;
  const long long rows = batches * heads * Lq;
  L.counters = 0;
  L.part_lse = align256(batches * heads * nqb * 4);
  L.part_o = L.part_lse + align256((long long)splits * rows * 4);
  L.total = L.part_o + (long long)splits * rows * 64 * 4;
  return L;
}

}  // namespace

// The launch behind every attention entry point: validates the arguments,
// encodes the TMA maps and launches one CTA per (batch, head, query block,
// split).  With splits > 1 the counters at the start of `scratch` are cleared
// on the stream first.
int attention_launch(const void* q, int64_t q_stride, const void* kv, int64_t kv_stride, int64_t k_col0,
                     int64_t v_col0, void* out, int64_t o_stride, int64_t batches, int64_t Lq, int64_t Lkv,
                     int64_t seg0_start, int64_t seg0_len, int64_t seg1_start, int64_t seg1_len, int32_t heads,
                     int32_t splits, int32_t lse_mode, float* lse, void* scratch, int64_t scratch_bytes,
                     void* stream) {
  if (batches < 0 || Lq < 0 || heads <= 0) return set_error(QVGGT_ERR_INVALID, "attention: bad shape");
  if (Lkv <= 0) return set_error(QVGGT_ERR_INVALID, "attention: Lkv must be > 0");
  if (seg0_start < 0 || seg0_len <= 0 || seg1_start < 0 || seg1_len < 0 || seg0_start + seg0_len > Lkv ||
      seg1_start + seg1_len > Lkv)
    return set_error(QVGGT_ERR_INVALID, "attention: key segments must lie inside [0, Lkv) and segment 0 be non-empty");
  if (lse_mode < 0 || lse_mode > 2) return set_error(QVGGT_ERR_INVALID, "attention: lse_mode must be 0, 1 or 2");
  if (lse_mode != 0 && lse == nullptr) return set_error(QVGGT_ERR_INVALID, "attention: lse_mode needs an lse buffer");
  if (q_stride % 8 || kv_stride % 8 || o_stride % 8 || k_col0 % 8 || v_col0 % 8)
    return set_error(QVGGT_ERR_ALIGN, "attention: strides and column offsets must be multiples of 8");
  if (!aligned16(q) || !aligned16(kv) || !aligned16(out) || (scratch && !aligned16(scratch)) ||
      (reinterpret_cast<uintptr_t>(lse) & 3))
    return set_error(QVGGT_ERR_ALIGN, "attention: tensors must be 16-byte aligned (lse 4-byte)");
  if (q_stride < heads * 64 || o_stride < heads * 64 || kv_stride < k_col0 + heads * 64 ||
      kv_stride < v_col0 + heads * 64)
    return set_error(QVGGT_ERR_INVALID, "attention: strides too small for the heads");
  const long long q_rows = batches * Lq, kv_rows = batches * Lkv;
  if (q_rows + 256 > 2147483647LL || kv_rows + 128 > 2147483647LL)
    return set_error(QVGGT_ERR_UNSUPPORTED, "attention: too many rows for 32-bit TMA coordinates");
  const long long nt0 = (seg0_len + 127) / 128, nt = nt0 + (seg1_len + 127) / 128;
  if (splits < 1 || splits > MAX_SPLITS || splits > nt)
    return set_error(QVGGT_ERR_INVALID, "attention: splits must be in 1..%d and at most the %lld key tiles", MAX_SPLITS,
                     nt);
  if (batches == 0 || Lq == 0) return QVGGT_OK;
  const ScratchLayout SL = scratch_layout(batches, Lq, heads, splits);
  if (splits > 1 && (scratch == nullptr || scratch_bytes < SL.total))
    return set_error(QVGGT_ERR_INVALID, "attention: %d splits need %lld bytes of scratch, got %lld", splits,
                     SL.total, (long long)scratch_bytes);
  const DeviceInfo& di = device_info();
  if (AttnSmem::TOTAL > di.max_smem_optin)
    return set_error(QVGGT_ERR_UNSUPPORTED, "attention: shared memory %d > %d", AttnSmem::TOTAL, di.max_smem_optin);

  CUtensorMap tmQ, tmK, tmV;
  {
    const uint64_t dims[3] = {64, (uint64_t)heads, (uint64_t)q_rows};
    const uint64_t strides[2] = {128, (uint64_t)q_stride * 2};
    const uint32_t box[3] = {64, 1, 128};
    int rc = encode_tmap(&tmQ, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, q, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    const uint64_t dims[3] = {64, (uint64_t)heads, (uint64_t)kv_rows};
    const uint64_t strides[2] = {128, (uint64_t)kv_stride * 2};
    const uint32_t box[3] = {64, 1, 128};
    const __half* kb = static_cast<const __half*>(kv) + k_col0;
    const __half* vb = static_cast<const __half*>(kv) + v_col0;
    int rc = encode_tmap(&tmK, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, kb, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = encode_tmap(&tmV, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, vb, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  AttnArgs a;
  a.batches = (int)batches;
  a.heads = heads;
  a.nqb = (int)((Lq + 255) / 256);
  a.splits = splits;
  a.nt0 = (int)nt0;
  a.nt = (int)nt;
  a.seg0_start = (int)seg0_start;
  a.seg0_len = (int)seg0_len;
  a.seg1_start = (int)seg1_start;
  a.seg1_len = (int)seg1_len;
  a.lse_mode = lse_mode;
  a.Lq = Lq;
  a.Lkv = Lkv;
  a.out = static_cast<__half*>(out);
  a.o_stride = o_stride;
  a.lse = lse;
  uint8_t* sc = static_cast<uint8_t*>(scratch);
  a.counters = splits > 1 ? reinterpret_cast<uint32_t*>(sc + SL.counters) : nullptr;
  a.part_lse = splits > 1 ? reinterpret_cast<float*>(sc + SL.part_lse) : nullptr;
  a.part_o = splits > 1 ? reinterpret_cast<float*>(sc + SL.part_o) : nullptr;
  a.scale_log2 = 0.125f * 1.4426950408889634f;
  a.ctl = make_ctl();
  const long long items = (long long)a.nqb * heads * batches;
  if (items * splits > 2147483647LL) return set_error(QVGGT_ERR_UNSUPPORTED, "attention: grid too large");
  // Share of exponentials computed on the FMA pipe (pairs per 8).  Measured
  // on B200 with the split S / PV issuers: 1 is fastest at the aggregator's
  // L = 43,968 (811 TFLOP/s vs 780 for 0 and 800 for 2); the QVGGT_ATTN_POLY
  // environment variable (0..4) overrides the default.
  static const int poly = [] {
    const char* e = getenv("QVGGT_ATTN_POLY");
    return (e && e[0] >= '0' && e[0] <= '4') ? e[0] - '0' : 1;
  }();
  const bool general = splits > 1 || lse_mode != 0;
  // general: one CTA per (item, split); plain: persistent, one CTA per SM
  // (the kernel's shared memory allows one) walking items gridDim.x apart
  const long long sms = device_info().num_sms;
  const long long grid = general ? items * splits : (items < sms ? items : sms);
  using Kfn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, AttnArgs);
  static const Kfn plain_fns[5] = {attn_fwd_kernel<0, false>, attn_fwd_kernel<1, false>, attn_fwd_kernel<2, false>,
                                   attn_fwd_kernel<3, false>, attn_fwd_kernel<4, false>};
  static const Kfn general_fns[5] = {attn_fwd_kernel<0, true>, attn_fwd_kernel<1, true>, attn_fwd_kernel<2, true>,
                                     attn_fwd_kernel<3, true>, attn_fwd_kernel<4, true>};
  const Kfn kfn = general ? general_fns[poly] : plain_fns[poly];
  static DeviceFlags attr_set[2][5];
  if (int rc = ensure_smem(attr_set[general][poly], kfn, AttnSmem::TOTAL, "cudaFuncSetAttribute(attention)"))
    return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (splits > 1) {
    if (int rc = check_cuda(cudaMemsetAsync(a.counters, 0, (size_t)a.nqb * heads * batches * 4, st),
                            "attention: clearing the split counters"))
      return rc;
  }
  int rc = check_cuda(launch_pdl(kfn, dim3((unsigned)grid), dim3(THREADS), AttnSmem::TOTAL, st, 1u, tmQ, tmK, tmV, a),
                      "attention launch");
  if (!rc) count_launch(1);
  return rc;
}

}  // namespace qv

using namespace qv;

extern "C" int qvggt_attention(const void* q, int64_t q_stride, const void* kv, int64_t kv_stride, int64_t k_col0,
                               int64_t v_col0, void* out, int64_t o_stride, int64_t batches, int64_t Lq, int64_t Lkv,
                               int32_t heads, void* stream) {
  return attention_launch(q, q_stride, kv, kv_stride, k_col0, v_col0, out, o_stride, batches, Lq, Lkv, 0, Lkv, 0, 0,
                          heads, 1, 0, nullptr, nullptr, 0, stream);
}

extern "C" int qvggt_attention_ex(const void* q, int64_t q_stride, const void* kv, int64_t kv_stride, int64_t k_col0,
                                  int64_t v_col0, void* out, int64_t o_stride, int64_t batches, int64_t Lq,
                                  int64_t Lkv, int64_t seg0_start, int64_t seg0_len, int64_t seg1_start,
                                  int64_t seg1_len, int32_t heads, int32_t splits, int32_t lse_mode, float* lse,
                                  void* scratch, int64_t scratch_bytes, void* stream) {
  return attention_launch(q, q_stride, kv, kv_stride, k_col0, v_col0, out, o_stride, batches, Lq, Lkv, seg0_start,
                          seg0_len, seg1_start, seg1_len, heads, splits, lse_mode, lse, scratch, scratch_bytes,
                          stream);
}

extern "C" int qvggt_attention_plan(int64_t batches, int64_t Lq, int64_t keys, int32_t heads, int32_t* splits,
                                    int64_t* scratch_bytes) {
  if (batches < 0 || Lq < 0 || keys <= 0 || heads <= 0 || !splits || !scratch_bytes)
    return set_error(QVGGT_ERR_INVALID, "attention_plan: bad arguments");
  const long long items = batches * heads * ((Lq + 255) / 256);
  const int nt = (int)std::min<long long>((keys + 127) / 128, 1 << 30);
  const int s = plan_splits(items, nt, device_info().num_sms);
  *splits = s;
  *scratch_bytes = scratch_layout(batches, Lq, heads, s).total;
  return QVGGT_OK;
}

extern "C" int qvggt_attention_scratch_bytes(int64_t batches, int64_t Lq, int32_t heads, int32_t splits,
                                             int64_t* scratch_bytes) {
  if (splits < 1 || splits > MAX_SPLITS)
    return set_error(QVGGT_ERR_INVALID, "attention_scratch_bytes: splits must be in 1..%d", MAX_SPLITS);
  if (batches < 0 || Lq < 0 || heads <= 0 || !scratch_bytes)
    return set_error(QVGGT_ERR_INVALID, "attention_scratch_bytes: bad arguments");
  *scratch_bytes = scratch_layout(batches, Lq, heads, splits).total;
  return QVGGT_OK;
}

// ------------------------------------------------------------------------
// Split-KV attention whose scratch lives in a fixed device array, for callers
// that may not allocate device memory: an allocator-less host runtime, code
// that runs while memory is being handed out by someone else (inside a memory
// pool's callback, a custom allocator, or a region where the owner forbids new
// allocations), or an integration that owns every byte of the GPU and cannot
// let a library call cudaMalloc behind its back.
namespace qv {
namespace {

// 64 MiB on every device that loads this library, held until the process
// exits.  It holds the split counters, the per-split log-sum-exps and the
// per-split fp32 output rows: splits * batches * heads * Lq rows of 260 bytes
// plus alignment (e.g. 2 splits of 16 heads x 5,496 queries, one rank of the
// 8-GPU aggregator, take 45.7 MB).
constexpr long long STATIC_SCRATCH_BYTES = 64LL << 20;
static __device__ __align__(256) uint8_t g_attn_static_scratch[STATIC_SCRATCH_BYTES];

// The array's device address, looked up once per device with that device
// current.  (In host code the array's name is a host-side stand-in, not an
// address a kernel may be given.)
std::once_flag g_static_once[kMaxDevices];
void* g_static_ptr[kMaxDevices] = {};
cudaError_t g_static_err[kMaxDevices] = {};

}  // namespace
}  // namespace qv

extern "C" int qvggt_attention_split_static(const void* q, int64_t q_stride, const void* kv, int64_t kv_stride,
                                            int64_t k_col0, int64_t v_col0, void* out, int64_t o_stride,
                                            int64_t batches, int64_t Lq, int64_t Lkv, int32_t heads, int32_t splits,
                                            void* stream) {
  int dev = -1;
  if (int rc = check_cuda(cudaGetDevice(&dev), "attention_split_static: cudaGetDevice")) return rc;
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(QVGGT_ERR_UNSUPPORTED, "attention_split_static: device %d beyond the %d this library tracks", dev,
                     kMaxDevices);
  if (splits < 1 || splits > MAX_SPLITS)
    return set_error(QVGGT_ERR_INVALID, "attention_split_static: splits must be in 1..%d", MAX_SPLITS);
  if (batches < 0 || Lq < 0 || heads <= 0) return set_error(QVGGT_ERR_INVALID, "attention_split_static: bad shape");
  const long long need = scratch_layout(batches, Lq, heads, splits).total;
  if (need > STATIC_SCRATCH_BYTES)
    return set_error(QVGGT_ERR_UNSUPPORTED,
                     "attention_split_static: %d splits of %lld batches x %d heads x %lld queries need %lld bytes of "
                     "scratch; the fixed array holds %lld (use fewer splits or qvggt_attention_ex with your own scratch)",
                     splits, (long long)batches, heads, (long long)Lq, need, STATIC_SCRATCH_BYTES);
  std::call_once(g_static_once[dev], [dev] {
    g_static_err[dev] = cudaGetSymbolAddress(&g_static_ptr[dev], g_attn_static_scratch);
  });
  if (g_static_err[dev] != cudaSuccess || g_static_ptr[dev] == nullptr)
    return set_error(QVGGT_ERR_CUDA, "attention_split_static: cudaGetSymbolAddress: %s",
                     cudaGetErrorString(g_static_err[dev]));
  return attention_launch(q, q_stride, kv, kv_stride, k_col0, v_col0, out, o_stride, batches, Lq, Lkv, 0, Lkv, 0, 0,
                          heads, splits, 0, nullptr, g_static_ptr[dev], STATIC_SCRATCH_BYTES, stream);
}
