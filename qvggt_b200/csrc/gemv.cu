// W4A16 GEMV for 1 <= m <= 16 rows: out[m, N] = x[m, K] . deq(W)^T (+ bias).
//
// HBM-bound on the packed weights (N*K/2 bytes).  One CTA of 4 warps per
// packed row g (output channels 4g..4g+3); each lane streams 16-byte chunks of
// the packed row with 128-bit loads (a 16-byte chunk = 32 nibbles of one
// channel over 32 consecutive k), dequantises them bit-exactly (same
// arithmetic as the GEMM and the reference's __hfma2), and accumulates
// x . w in fp32.  Partial sums are reduced with warp shuffles, then across the
// 4 warps through shared memory.
#include "host.hpp"

namespace qv {
namespace {

template <int MT, int MAXIT>
__global__ void __launch_bounds__(128) gemv_w4_kernel(const __half* __restrict__ x, const uint16_t* __restrict__ qw,
                                                      const __half* __restrict__ scales,
                                                      const __half* __restrict__ zeros, const __half* __restrict__ bias,
                                                      __half* __restrict__ out, int m, int N, int K, int G) {
  __shared__ float red[4][4][MT];
  const int g = blockIdx.x;           // packed row
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint8_t* row = reinterpret_cast<const uint8_t*>(qw + (size_t)g * K);
  const int row_bytes = K * 2;
  float acc[MT];
#pragma unroll
  for (int i = 0; i < MT; ++i) acc[i] = 0.f;

  // Byte offset of this lane's chunk: ((it*4 + warp)*32 + lane)*16.  Within a
  // 128-byte k-chunk c: channel i = (off%128)/32, half h = (off%32)/16.
  const int ci = (lane & 7) >> 1;   // constant over iterations (stride is a multiple of 128 B)
  const int h = lane & 1;
  const __half2 magic = __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400));
  // Issue every weight (and scale / zero) load of this thread before any math,
  // so up to MAXIT 16-byte loads per thread are in flight at once.
  uint4 wvs[MAXIT];
  __half ss[MAXIT], zs[MAXIT];
  const int off0 = (warp * 32 + lane) * 16;
#pragma unroll
  for (int it = 0; it < MAXIT; ++it) {
    const int off = off0 + it * 128 * 16;
    if (off < row_bytes) {
      wvs[it] = __ldg(reinterpret_cast<const uint4*>(row + off));
      const int grp = (64 * (off >> 7) + 32 * h) / G;
      ss[it] = scales[(size_t)grp * N + 4 * g + ci];
      zs[it] = zeros[(size_t)grp * N + 4 * g + ci];
    }
  }
#pragma unroll
  for (int it = 0; it < MAXIT; ++it) {
    const int off = off0 + it * 128 * 16;
    if (off >= row_bytes) break;
    const int c = off >> 7;
    const int k0 = 64 * c + 32 * h;
    const uint4 wv = wvs[it];
    const __half2 s2 = __half2half2(ss[it]), z2 = __half2half2(zs[it]);
    const uint32_t xs[4] = {wv.x, wv.y, wv.z, wv.w};
    // w[q][u] covers k = k0 + 8q + 2u, +1
    float2 w[4][4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        uint32_t t;
        const uint32_t src = xs[u] >> (4 * q);
        asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(t) : "r"(src), "r"(0x000F000Fu), "r"(0x64006400u));
        __half2 hq = __hsub2(*reinterpret_cast<__half2*>(&t), magic);
        w[q][u] = __half22float2(__hfma2(hq, s2, z2));
      }
    }
#pragma unroll
    for (int r = 0; r < MT; ++r) {
      if (r < m) {
        const uint4* xp = reinterpret_cast<const uint4*>(x + (size_t)r * K + k0);
        float a = acc[r];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 xv = __ldg(xp + q);
          const uint32_t xu[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            float2 xf = unpack_half2(xu[u]);
            a = fmaf(xf.x, w[q][u].x, a);
            a = fmaf(xf.y, w[q][u].y, a);
          }
        }
        acc[r] = a;
      }
    }
  }
  // Lanes sharing channel ci: lane%8 in {2ci, 2ci+1}, lane/8 in 0..3.
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
    for (int r = 0; r < MT; ++r) red[warp][ci][r] = acc[r];
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < 4 * m; idx += blockDim.x) {
    const int r = idx >> 2, ch = idx & 3;
    float v = red[0][ch][r] + red[1][ch][r] + red[2][ch][r] + red[3][ch][r];
    const int n = 4 * g + ch;
    if (r < MT) {
      float y = round_f16(v);
      if (bias) y = y + __half2float(bias[n]);
      out[(size_t)r * N + n] = __float2half_rn(y);
    }
  }
}

}  // namespace
}  // namespace qv

using namespace qv;

extern "C" int qvggt_w4a16_gemv(const void* in_feats, const void* qweight, const void* scales,
                                const void* scaled_zeros, const void* bias, void* out, int64_t m, int64_t N,
                                int64_t K, int64_t gpad, int32_t group_size, void* stream) {
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
  const dim3 grid((unsigned)(N / 4)), block(128);
  auto args = [&](auto kfn) {
    kfn<<<grid, block, 0, st>>>(static_cast<const __half*>(in_feats), static_cast<const uint16_t*>(qweight),
                                static_cast<const __half*>(scales), static_cast<const __half*>(scaled_zeros),
                                static_cast<const __half*>(bias), static_cast<__half*>(out), (int)m, (int)N, (int)K,
                                group_size);
  };
  // 16-byte chunks per thread: a packed row is 2K bytes, a CTA covers 2 KB per pass
  const int iters = (int)((K * 2 + 2047) / 2048);
  auto by_m = [&](auto mt) {
    constexpr int MT = decltype(mt)::value;
    if (iters <= 1) args(gemv_w4_kernel<MT, 1>);
    else if (iters <= 2) args(gemv_w4_kernel<MT, 2>);
    else if (iters <= 4) args(gemv_w4_kernel<MT, 4>);
    else if (iters <= 8) args(gemv_w4_kernel<MT, 8>);
    else args(gemv_w4_kernel<MT, 16>);
  };
  if (K > 16384) return set_error(QVGGT_ERR_UNSUPPORTED, "gemv: K=%lld > 16384", (long long)K);
  if (m <= 1) by_m(std::integral_constant<int, 1>());
  else if (m <= 2) by_m(std::integral_constant<int, 2>());
  else if (m <= 4) by_m(std::integral_constant<int, 4>());
  else if (m <= 8) by_m(std::integral_constant<int, 8>());
  else by_m(std::integral_constant<int, 16>());
  int rc = check_cuda(cudaGetLastError(), "gemv launch");
  if (rc == QVGGT_OK) count_launch(1);
  return rc;
}
