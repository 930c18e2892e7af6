// Memory-bound row kernels: LayerNorm (fp16 -> fp16), LayerNorm + per-token
// int8 quantisation, per-token int8 quantisation, tanh-GELU + quantisation.
//
// One warp per row, the whole row held in registers (16-byte vector loads and
// stores, coalesced across the warp), warp-shuffle reductions only: every
// byte is read once from HBM and written once.
#include "host.hpp"

namespace qv {
namespace {

constexpr int ROWS_PER_BLOCK = 8;  // warps per CTA

// Load CH 16-byte chunks (8 fp16 each) of a row: chunk j of lane l sits at
// element (j*32 + l)*8, so each warp-wide load is one contiguous 512-byte span.
template <int CH>
__device__ __forceinline__ void load_row(const __half* row, int lane, float (&v)[CH * 8]) {
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    uint4 u = *reinterpret_cast<const uint4*>(row + (j * 32 + lane) * 8);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      float2 f = unpack_half2(w[t]);
      v[j * 8 + 2 * t] = f.x;
      v[j * 8 + 2 * t + 1] = f.y;
    }
  }
}

template <int CH>
__device__ __forceinline__ void load_vec(const __half* p, int lane, float (&v)[CH * 8]) {
  load_row<CH>(p, lane, v);
}

// ---------------------------------------------------------------- LayerNorm
template <int CH>
__global__ void __launch_bounds__(ROWS_PER_BLOCK * 32) layernorm_kernel(const __half* __restrict__ x,
                                                                        const __half* __restrict__ w,
                                                                        const __half* __restrict__ b,
                                                                        __half* __restrict__ y, long long T, float eps) {
  pdl_wait();
  pdl_trigger();
  constexpr int H = CH * 256;
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * ROWS_PER_BLOCK + (threadIdx.x >> 5);
  if (row >= T) return;
  float v[CH * 8];
  load_row<CH>(x + row * H, lane, v);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < CH * 8; ++i) s += v[i];
  const float mean = warp_sum(s) * (1.0f / H);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < CH * 8; ++i) {
    const float d = v[i] - mean;
    q = fmaf(d, d, q);
  }
  const float rstd = rsqrtf(warp_sum(q) * (1.0f / H) + eps);
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    const uint4 wu = __ldg(reinterpret_cast<const uint4*>(w + (j * 32 + lane) * 8));
    const uint4 bu = __ldg(reinterpret_cast<const uint4*>(b + (j * 32 + lane) * 8));
    const uint32_t wa[4] = {wu.x, wu.y, wu.z, wu.w}, ba[4] = {bu.x, bu.y, bu.z, bu.w};
    uint32_t o[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int i = j * 8 + 2 * t;
      const float2 gw = unpack_half2(wa[t]), gb = unpack_half2(ba[t]);
      o[t] = pack_half2(fmaf((v[i] - mean) * rstd, gw.x, gb.x), fmaf((v[i + 1] - mean) * rstd, gw.y, gb.y));
    }
    *reinterpret_cast<uint4*>(y + row * H + (j * 32 + lane) * 8) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// ------------------------------------------------- LayerNorm + int8 quantisation
// Follows generalLayerNorm (w8a8/layernorm.cu:20-151): variance as
// E[x^2] - E[x]^2, rsqrt, fp32 LN; per-token: amax over the fp16-rounded LN
// values (floor half(1e-6)), int8 = rni_sat(fp32 LN * 127/amax), scale =
// half(amax/127); per-tensor: int8 = rni_sat(float(half(LN)) * scale).
template <int CH, bool PER_TOKEN>
__global__ void __launch_bounds__(ROWS_PER_BLOCK * 32) layernorm_quant_kernel(
    const __half* __restrict__ x, const __half* __restrict__ w, const __half* __restrict__ b,
    int8_t* __restrict__ out, __half* __restrict__ scale, long long T, float eps) {
  pdl_wait();
  pdl_trigger();
  constexpr int H = CH * 256;
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * ROWS_PER_BLOCK + (threadIdx.x >> 5);
  if (row >= T) return;
  float v[CH * 8];
  load_row<CH>(x + row * H, lane, v);
  float s = 0.f, s2 = 0.f;
#pragma unroll
  for (int i = 0; i < CH * 8; ++i) {
    s += v[i];
    s2 = fmaf(v[i], v[i], s2);
  }
  const float mean = warp_sum(s) / H;
  const float var = warp_sum(s2) / H - mean * mean;
  const float rs = rsqrtf(var + eps);
  float gw[CH * 8], gb[CH * 8];
  load_vec<CH>(w, lane, gw);
  if (PER_TOKEN) {
    load_vec<CH>(b, lane, gb);
  }
  float ln[CH * 8];
#pragma unroll
  for (int i = 0; i < CH * 8; ++i) {
    ln[i] = (v[i] - mean) * rs * gw[i];
    if (PER_TOKEN) ln[i] += gb[i];
  }
  float qs;
  if (PER_TOKEN) {
    float amax = __half2float(__float2half_rn(1e-6f));
#pragma unroll
    for (int i = 0; i < CH * 8; ++i) amax = fmaxf(amax, fabsf(round_f16(ln[i])));
    amax = warp_max(amax);
    qs = 127.f / amax;
    if (lane == 0) scale[row] = __float2half_rn(amax / 127.f);
  } else {
    qs = __half2float(scale[0]);
#pragma unroll
    for (int i = 0; i < CH * 8; ++i) ln[i] = round_f16(ln[i]);
  }
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    uint32_t o[2];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      uint32_t pk = 0;
#pragma unroll
      for (int e = 0; e < 4; ++e)
        pk |= (uint32_t)(uint8_t)f32_to_s8_rni_sat(ln[j * 8 + 4 * t + e] * qs) << (8 * e);
      o[t] = pk;
    }
    *reinterpret_cast<uint2*>(out + row * H + (j * 32 + lane) * 8) = make_uint2(o[0], o[1]);
  }
}

// ------------------------------------------------------------- invoke_quant
// quant_kernel (w8a8/quantization.cu:41-78): amax = max|x| (start 0),
// scale = half(amax / 127), int8 = rni_sat(x * (127 / amax)).
template <int CH>
__global__ void __launch_bounds__(ROWS_PER_BLOCK * 32) quant_kernel(const __half* __restrict__ x,
                                                                    int8_t* __restrict__ out,
                                                                    __half* __restrict__ scale, long long T) {
  pdl_wait();
  pdl_trigger();
  constexpr int H = CH * 256;
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * ROWS_PER_BLOCK + (threadIdx.x >> 5);
  if (row >= T) return;
  float v[CH * 8];
  load_row<CH>(x + row * H, lane, v);
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < CH * 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
  amax = warp_max(amax);
  const float qs = 127.f / amax;
  if (lane == 0) scale[row] = __float2half_rn(amax / 127.f);
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    uint32_t o[2];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      uint32_t pk = 0;
#pragma unroll
      for (int e = 0; e < 4; ++e) pk |= (uint32_t)(uint8_t)f32_to_s8_rni_sat(v[j * 8 + 4 * t + e] * qs) << (8 * e);
      o[t] = pk;
    }
    *reinterpret_cast<uint2*>(out + row * H + (j * 32 + lane) * 8) = make_uint2(o[0], o[1]);
  }
}

// ----------------------------------------------------------- gelu_and_quant
// gelu_and_quant_kernel (w8a8/act.cu:22-74), per-token path: tanh-GELU in fp16
// arithmetic, tmp written, amax over (t > 1e-4 ? t : -t), scale = half(amax/127),
// int8 = rni_sat(float(half(127/amax) * t)).
__device__ __forceinline__ __half gelu_fast_h(__half x) {
  const __half f = x;
  const __half a = __hmul(f, __float2half_rn(0.79788456f));
  const __half bq = __hmul(__float2half_rn(0.044715f), f);
  // the reference's half `1 + bq * x` is contracted by nvcc into one fma
  const __half d = __hfma(bq, x, __float2half_rn(1.0f));
  const __half e = __hmul(a, d);
  const __half t = __float2half_rn(tanhf(__half2float(e)));
  return __hmul(__hmul(__float2half_rn(0.5f), x), __hadd(__float2half_rn(1.0f), t));
}

template <int CH>
__global__ void __launch_bounds__(ROWS_PER_BLOCK * 32) gelu_quant_kernel(const __half* __restrict__ x,
                                                                         int8_t* __restrict__ out,
                                                                         __half* __restrict__ scale,
                                                                         __half* __restrict__ tmp, long long T) {
  pdl_wait();
  pdl_trigger();
  constexpr int H = CH * 256;
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * ROWS_PER_BLOCK + (threadIdx.x >> 5);
  if (row >= T) return;
  // GELU outputs kept as packed half2 words (an array of 16-bit halves was
  // placed in local memory)
  uint32_t t2[CH * 4];
  float amax = 0.f;
  const __half zero = __float2half_rn(0.0001f);
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    uint4 u = *reinterpret_cast<const uint4*>(x + row * H + (j * 32 + lane) * 8);
    const uint32_t xw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const __half2 hx = *reinterpret_cast<const __half2*>(&xw[e]);
      const __half g0 = gelu_fast_h(__low2half(hx)), g1 = gelu_fast_h(__high2half(hx));
      const __half2 g = __halves2half2(g0, g1);
      t2[j * 4 + e] = *reinterpret_cast<const uint32_t*>(&g);
      const __half a0 = __hgt(g0, zero) ? g0 : __hneg(g0);
      const __half a1 = __hgt(g1, zero) ? g1 : __hneg(g1);
      amax = fmaxf(amax, __half2float(a0));
      amax = fmaxf(amax, __half2float(a1));
    }
    *reinterpret_cast<uint4*>(tmp + row * H + (j * 32 + lane) * 8) =
        make_uint4(t2[j * 4], t2[j * 4 + 1], t2[j * 4 + 2], t2[j * 4 + 3]);
  }
  amax = warp_max(amax);
  if (lane == 0) scale[row] = __float2half_rn(amax / 127.f);
  const __half hs = __float2half_rn(127.f / amax);
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    uint32_t o[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      uint32_t pk = 0;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const __half2 g = *reinterpret_cast<const __half2*>(&t2[j * 4 + 2 * q + e]);
        pk |= (uint32_t)(uint8_t)f32_to_s8_rni_sat(__half2float(__hmul(hs, __low2half(g)))) << (16 * e);
        pk |= (uint32_t)(uint8_t)f32_to_s8_rni_sat(__half2float(__hmul(hs, __high2half(g)))) << (16 * e + 8);
      }
      o[q] = pk;
    }
    *reinterpret_cast<uint2*>(out + row * H + (j * 32 + lane) * 8) = make_uint2(o[0], o[1]);
  }
}

inline dim3 rows_grid(long long T) { return dim3((unsigned)((T + ROWS_PER_BLOCK - 1) / ROWS_PER_BLOCK)); }

int check_rows(const char* what, int64_t T, int64_t H, const void* a, const void* b) {
  if (T < 0) return set_error(QVGGT_ERR_INVALID, "%s: tokens < 0", what);
  if (H <= 0 || H % 256 || H > 4096)
    return set_error(QVGGT_ERR_UNSUPPORTED, "%s: hidden=%lld must be a multiple of 256 up to 4096", what,
                     (long long)H);
  if (!aligned16(a) || !aligned16(b)) return set_error(QVGGT_ERR_ALIGN, "%s: tensors must be 16-byte aligned", what);
  return QVGGT_OK;
}

#define QV_DISPATCH_CH(H, ...)                   \
  switch ((H) / 256) {                           \
    case 1: { constexpr int CH = 1; __VA_ARGS__; break; } \
    case 2: { constexpr int CH = 2; __VA_ARGS__; break; } \
    case 3: { constexpr int CH = 3; __VA_ARGS__; break; } \
    case 4: { constexpr int CH = 4; __VA_ARGS__; break; } \
    case 8: { constexpr int CH = 8; __VA_ARGS__; break; } \
    case 12: { constexpr int CH = 12; __VA_ARGS__; break; } \
    case 16: { constexpr int CH = 16; __VA_ARGS__; break; } \
    default: return set_error(QVGGT_ERR_UNSUPPORTED, "hidden=%lld not instantiated", (long long)(H)); \
  }

#define QV_DISPATCH_CH_SMALL(H, ...)             \
  switch ((H) / 256) {                           \
    case 1: { constexpr int CH = 1; __VA_ARGS__; break; } \
    case 2: { constexpr int CH = 2; __VA_ARGS__; break; } \
    case 3: { constexpr int CH = 3; __VA_ARGS__; break; } \
    case 4: { constexpr int CH = 4; __VA_ARGS__; break; } \
    case 8: { constexpr int CH = 8; __VA_ARGS__; break; } \
    default: return set_error(QVGGT_ERR_UNSUPPORTED, "hidden=%lld not instantiated", (long long)(H)); \
  }

}  // namespace
}  // namespace qv

using namespace qv;

extern "C" {

int qvggt_layernorm(const void* in, const void* gamma, const void* beta, void* out, int64_t tokens, int64_t hidden,
                    float eps, void* stream) {
  int rc = check_rows("layernorm", tokens, hidden, in, out);
  if (rc) return rc;
  if (hidden > 2048) return set_error(QVGGT_ERR_UNSUPPORTED, "layernorm: hidden=%lld > 2048", (long long)hidden);
  if (!gamma || !beta) return set_error(QVGGT_ERR_INVALID, "layernorm: gamma and beta required");
  if (tokens == 0) return QVGGT_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t err = cudaSuccess;
  QV_DISPATCH_CH_SMALL(hidden, err = launch_pdl(layernorm_kernel<CH>, dim3(rows_grid(tokens)), dim3(ROWS_PER_BLOCK * 32),
                                                0, st, 1u, static_cast<const __half*>(in),
                                                static_cast<const __half*>(gamma), static_cast<const __half*>(beta),
                                                static_cast<__half*>(out), (long long)tokens, eps));
  rc = check_cuda(err, "layernorm launch");
  if (!rc) count_launch(1);
  return rc;
}

int qvggt_layernorm_quant(int8_t* out, const void* in, const void* gamma, const void* beta, void* scale_io,
                          int64_t tokens, int64_t hidden, float eps, int32_t per_token, void* stream) {
  int rc = check_rows("layernorm_quant", tokens, hidden, in, out);
  if (rc) return rc;
  if (hidden > 2048) return set_error(QVGGT_ERR_UNSUPPORTED, "layernorm_quant: hidden=%lld > 2048", (long long)hidden);
  if (!gamma || !scale_io || (per_token && !beta))
    return set_error(QVGGT_ERR_INVALID, "layernorm_quant: gamma, scale (and beta per-token) required");
  if (tokens == 0) return QVGGT_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t err = cudaSuccess;
  const dim3 grid(rows_grid(tokens)), block(ROWS_PER_BLOCK * 32);
  if (per_token) {
    QV_DISPATCH_CH_SMALL(hidden, err = launch_pdl(layernorm_quant_kernel<CH, true>, grid, block, 0, st, 1u,
                                                  static_cast<const __half*>(in), static_cast<const __half*>(gamma),
                                                  static_cast<const __half*>(beta), out,
                                                  static_cast<__half*>(scale_io), (long long)tokens, eps));
  } else {
    QV_DISPATCH_CH_SMALL(hidden, err = launch_pdl(layernorm_quant_kernel<CH, false>, grid, block, 0, st, 1u,
                                                  static_cast<const __half*>(in), static_cast<const __half*>(gamma),
                                                  static_cast<const __half*>(nullptr), out,
                                                  static_cast<__half*>(scale_io), (long long)tokens, eps));
  }
  rc = check_cuda(err, "layernorm_quant launch");
  if (!rc) count_launch(1);
  return rc;
}

int qvggt_invoke_quant(int8_t* out, const void* in, void* scale, int64_t tokens, int64_t hidden, void* stream) {
  int rc = check_rows("invoke_quant", tokens, hidden, in, out);
  if (rc) return rc;
  if (tokens == 0) return QVGGT_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t err = cudaSuccess;
  QV_DISPATCH_CH(hidden, err = launch_pdl(quant_kernel<CH>, dim3(rows_grid(tokens)), dim3(ROWS_PER_BLOCK * 32), 0, st,
                                          1u, static_cast<const __half*>(in), out, static_cast<__half*>(scale),
                                          (long long)tokens));
  rc = check_cuda(err, "invoke_quant launch");
  if (!rc) count_launch(1);
  return rc;
}

int qvggt_gelu_quant(int8_t* out, const void* in, void* scale, void* tmp, int64_t tokens, int64_t d, void* stream) {
  int rc = check_rows("gelu_quant", tokens, d, in, out);
  if (rc) return rc;
  if (!aligned16(tmp)) return set_error(QVGGT_ERR_ALIGN, "gelu_quant: tmp must be 16-byte aligned");
  if (tokens == 0) return QVGGT_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t err = cudaSuccess;
  QV_DISPATCH_CH(d, err = launch_pdl(gelu_quant_kernel<CH>, dim3(rows_grid(tokens)), dim3(ROWS_PER_BLOCK * 32), 0, st,
                                     1u, static_cast<const __half*>(in), out, static_cast<__half*>(scale),
                                     static_cast<__half*>(tmp), (long long)tokens));
  rc = check_cuda(err, "gelu_quant launch");
  if (!rc) count_launch(1);
  return rc;
}

}  // extern "C"
