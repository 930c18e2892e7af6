// W4A16 GEMV for 1 <= m <= 16 rows: out[m, N] = x[m, K] . deq(W)^T (+ bias).
//
// HBM-bound on the packed weights (N*K/2 bytes), and at the sizes it runs on
// (a few MB) bound just as much by how fast all of them are in flight and how
// well the dequantisation's dependent ALU chains are interleaved.  Four warps
// per packed row g (output channels 4g..4g+3), four rows per 512-thread CTA
// (N = 4096 is 256 CTAs, two resident per SM, all in flight at once): each
// lane issues 4 128-bit loads of its quarter of the row (a 16-byte chunk = 32
// nibbles of one channel over 32 consecutive k) plus their scales and zeros
// before using any, x is staged once per CTA in shared memory by asynchronous
// copies issued first, and each channel's sum is reduced with three shuffles
// within a warp and then over the row's four warps in shared memory.
// Weights are dequantised bit-exactly (same arithmetic as the GEMM and the
// reference's __hfma2); x . w is formed over each run of 8 consecutive k with
// fp16x2 FMAs and that partial is added into an fp32 accumulator (the
// reference's GEMV accumulates every product of a thread in fp16; a product
// is exact when x is one-hot).  The bf16 form (BF) dequantises with the bf16
// magic pattern and bf16x2 FMA (dequantize.cuh:53-90) and forms x . w in fp32
// (bf16 widens to fp32 exactly; the reference accumulates in bf16).
#include <type_traits>

#include "host.hpp"

namespace qv {
namespace {

constexpr int GEMV_ROWS = 4;              // packed rows per CTA
constexpr int GEMV_WARPS = 4 * GEMV_ROWS; // four warps per packed row
constexpr int GEMV_BATCH = 4;             // 16-byte chunks per lane in flight
constexpr int GEMV_XS_MAX = 32768;        // x staged in shared memory up to this many bytes

__device__ __forceinline__ void cp_async16(uint32_t dst_smem, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst_smem), "l"(src) : "memory");
}

template <int MT, bool XS, bool BF>
__global__ void __launch_bounds__(GEMV_WARPS * 32, MT == 1 ? 2 : 1) gemv_w4_kernel(
    const void* __restrict__ x_, const uint16_t* __restrict__ qw, const void* __restrict__ scales_,
    const void* __restrict__ zeros_, const void* __restrict__ bias_, void* __restrict__ out_, int m, int N, int K,
    int G) {
  using T = std::conditional_t<BF, __nv_bfloat16, __half>;
  using T2 = std::conditional_t<BF, __nv_bfloat162, __half2>;
  const T* x = static_cast<const T*>(x_);
  const T* scales = static_cast<const T*>(scales_);
  const T* zeros = static_cast<const T*>(zeros_);
  const T* bias = static_cast<const T*>(bias_);
  T* out = static_cast<T*>(out_);
  extern __shared__ __align__(16) uint8_t x_smem_raw[];   // XS: x [m, K]
  T* x_smem = reinterpret_cast<T*>(x_smem_raw);
  pdl_wait();
  pdl_trigger();
  __shared__ float red[GEMV_ROWS][4][4][MT];          // [row][quarter][channel][m]
  if constexpr (XS) {
    const int chunks = m * K / 8;
    for (int q = threadIdx.x; q < chunks; q += blockDim.x) cp_async16(smem_u32(x_smem + 8 * q), x + 8 * q);
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rw = warp >> 2, wq = warp & 3;            // row of the CTA, quarter of the row
  const int g = blockIdx.x * GEMV_ROWS + rw;          // packed row of this warp
  const bool active = g < N / 4;
  const uint8_t* row = reinterpret_cast<const uint8_t*>(qw + (size_t)(active ? g : 0) * K);
  const int row_bytes = K * 2;
  // Chunk it of a batch sits at byte base + ((it*4 + wq)*32 + lane)*16; within
  // a 128-byte k-chunk c that is channel ci = (lane%8)/2, half h = lane%2.
  const int ci = (lane & 7) >> 1;
  const int h = lane & 1;
  const uint32_t magic_u = BF ? 0x43004300u : 0x64006400u;
  const T2 magic = *reinterpret_cast<const T2*>(&magic_u);
  float acc[MT];
#pragma unroll
  for (int r = 0; r < MT; ++r) acc[r] = 0.f;
  for (int base = 0; base < row_bytes; base += GEMV_BATCH * 2048) {
    uint4 wvs[GEMV_BATCH];
    T ss[GEMV_BATCH], zs[GEMV_BATCH];
#pragma unroll
    for (int it = 0; it < GEMV_BATCH; ++it) {
      const int off = base + ((it * 4 + wq) * 32 + lane) * 16;
      if (active && off < row_bytes) {
        wvs[it] = __ldg(reinterpret_cast<const uint4*>(row + off));
        const int grp = (64 * (off >> 7) + 32 * h) / G;
        ss[it] = scales[(size_t)grp * N + 4 * g + ci];
        zs[it] = zeros[(size_t)grp * N + 4 * g + ci];
      }
    }
    if (XS && base == 0) {
      asm volatile("cp.async.wait_all;" ::: "memory");
      __syncthreads();
    }
    if (!active) continue;
#pragma unroll
    for (int it = 0; it < GEMV_BATCH; ++it) {
      const int off = base + ((it * 4 + wq) * 32 + lane) * 16;
      if (off >= row_bytes) break;
      const int k0 = 64 * (off >> 7) + 32 * h;
      const uint4 wv = wvs[it];
      const T2 s2 = T2(ss[it], ss[it]), z2 = T2(zs[it], zs[it]);
      const uint32_t xw[4] = {wv.x, wv.y, wv.z, wv.w};
      // w[q][u] (dequantised pair) covers k = k0 + 8q + 2u, +1
      T2 w[4][4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint32_t t;
          const uint32_t src = xw[u] >> (4 * q);
          asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(t) : "r"(src), "r"(0x000F000Fu), "r"(magic_u));
          const T2 hq = __hsub2(*reinterpret_cast<T2*>(&t), magic);
          w[q][u] = __hfma2(hq, s2, z2);
        }
      }
#pragma unroll
      for (int r = 0; r < MT; ++r) {
        if (r < m) {
          const uint4* xp = reinterpret_cast<const uint4*>((XS ? x_smem : x) + (size_t)r * K + k0);
          float a = acc[r];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 xv = XS ? xp[q] : __ldg(xp + q);
            const uint32_t xu[4] = {xv.x, xv.y, xv.z, xv.w};
            if constexpr (BF) {
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const float2 xf = unpack_bf162(xu[u]);
                const float2 wf = unpack_bf162(*reinterpret_cast<const uint32_t*>(&w[q][u]));
                a = fmaf(xf.x, wf.x, a);
                a = fmaf(xf.y, wf.y, a);
              }
            } else {
              // x . w over these 8 k in fp16x2, then one fp32 add per half
              __half2 p = __hmul2(*reinterpret_cast<const __half2*>(&xu[0]), w[q][0]);
#pragma unroll
              for (int u = 1; u < 4; ++u) p = __hfma2(*reinterpret_cast<const __half2*>(&xu[u]), w[q][u], p);
              const float2 pf = __half22float2(p);
              a += pf.x + pf.y;
            }
          }
          acc[r] = a;
        }
      }
    }
  }
  // lanes holding channel ci: lane%8 in {2ci, 2ci+1}, lane/8 in 0..3
#pragma unroll
  for (int r = 0; r < MT; ++r) {
    float v = acc[r];
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 8);
    v += __shfl_xor_sync(0xffffffffu, v, 16);
    acc[r] = v;
  }
  if (lane < 8 && (lane & 1) == 0) {
#pragma unroll
    for (int r = 0; r < MT; ++r) red[rw][wq][ci][r] = acc[r];
  }
  __syncthreads();
  // the row's four quarters, summed in a fixed order
  for (int idx = threadIdx.x; idx < GEMV_ROWS * 4 * m; idx += blockDim.x) {
    const int r = idx % m, ch = (idx / m) % 4, rr = idx / (4 * m);
    const int gg = blockIdx.x * GEMV_ROWS + rr;
    if (gg >= N / 4 || r >= MT) continue;
    const float v = red[rr][0][ch][r] + red[rr][1][ch][r] + red[rr][2][ch][r] + red[rr][3][ch][r];
    const int n = 4 * gg + ch;
    if constexpr (BF) {
      float y = round_bf16(v);
      if (bias) y = y + __bfloat162float(bias[n]);
      out[(size_t)r * N + n] = __float2bfloat16_rn(y);
    } else {
      float y = round_f16(v);
      if (bias) y = y + __half2float(bias[n]);
      out[(size_t)r * N + n] = __float2half_rn(y);
    }
  }
}

}  // namespace
}  // namespace qv

using namespace qv;

namespace {

int gemv_launch(bool bf16, const void* in_feats, const void* qweight, const void* scales, const void* scaled_zeros,
                const void* bias, void* out, int64_t m, int64_t N, int64_t K, int64_t gpad, int32_t group_size,
                void* stream) {
  if (m < 1 || m > 16) return set_error(QVGGT_ERR_UNSUPPORTED, "gemv: m=%lld must be in 1..16", (long long)m);
  if (N <= 0 || N % 4 || K <= 0 || K % 64)
    return set_error(QVGGT_ERR_INVALID, "gemv: N=%lld must be a multiple of 4, K=%lld of 64", (long long)N,
                     (long long)K);
  if (group_size <= 0 || group_size % 32 || K % group_size)
    return set_error(QVGGT_ERR_UNSUPPORTED, "gemv: group_size=%d must be a multiple of 32 dividing K", group_size);
  if (gpad < K / group_size) return set_error(QVGGT_ERR_INVALID, "gemv: scale table has too few groups");
  if (!aligned16(in_feats) || !aligned16(qweight))
    return set_error(QVGGT_ERR_ALIGN, "gemv: in_feats / qweight must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)((N / 4 + GEMV_ROWS - 1) / GEMV_ROWS)), block(GEMV_WARPS * 32);
  // x staged in shared memory when it fits the default 48 KB with room to spare
  const int xs_bytes = (int)(m * K * 2);
  const bool xs = xs_bytes <= GEMV_XS_MAX;
  cudaError_t err = cudaSuccess;
  auto args = [&](auto kfn) {
    err = launch_pdl(kfn, grid, block, xs ? xs_bytes : 0, st, 1u, in_feats, static_cast<const uint16_t*>(qweight),
                     scales, scaled_zeros, bias, out, (int)m, (int)N, (int)K, (int)group_size);
  };
  auto by_m = [&](auto mt) {
    constexpr int MT = decltype(mt)::value;
    if (bf16) {
      if (xs) args(gemv_w4_kernel<MT, true, true>);
      else args(gemv_w4_kernel<MT, false, true>);
    } else {
      if (xs) args(gemv_w4_kernel<MT, true, false>);
      else args(gemv_w4_kernel<MT, false, false>);
    }
  };
  if (K > 16384) return set_error(QVGGT_ERR_UNSUPPORTED, "gemv: K=%lld > 16384", (long long)K);
  if (m <= 1) by_m(std::integral_constant<int, 1>());
  else if (m <= 2) by_m(std::integral_constant<int, 2>());
  else if (m <= 4) by_m(std::integral_constant<int, 4>());
  else if (m <= 8) by_m(std::integral_constant<int, 8>());
  else by_m(std::integral_constant<int, 16>());
  int rc = check_cuda(err, "gemv launch");
  if (rc == QVGGT_OK) count_launch(1);
  return rc;
}

}  // namespace

extern "C" int qvggt_w4a16_gemv(const void* in_feats, const void* qweight, const void* scales,
                                const void* scaled_zeros, const void* bias, void* out, int64_t m, int64_t N,
                                int64_t K, int64_t gpad, int32_t group_size, void* stream) {
  return gemv_launch(false, in_feats, qweight, scales, scaled_zeros, bias, out, m, N, K, gpad, group_size, stream);
}

extern "C" int qvggt_w4a16_gemv_bf16(const void* in_feats, const void* qweight, const void* scales,
                                     const void* scaled_zeros, const void* bias, void* out, int64_t m, int64_t N,
                                     int64_t K, int64_t gpad, int32_t group_size, void* stream) {
  return gemv_launch(true, in_feats, qweight, scales, scaled_zeros, bias, out, m, N, K, gpad, group_size, stream);
}
