// Patch embedding helpers for the DINOv2 ViT-L/14 front of the aggregator.
//
// patchify_kernel: images fp16 [S, 3, H, W] in [0, 1] -> normalised patches
//   fp16 [S * (H/p) * (W/p), k_pad] (column c*p*p + ky*p + kx, zero padding up
//   to k_pad), so the 14x14/stride-14 convolution becomes a GEMM on the
//   tcgen05 kernel.  Normalisation (x - mean_c) / std_c rounds to fp16 after
//   the subtraction and after the division, as the eager fp16 model does.
// assemble_kernel: builds token rows [S, P, C] from per-frame special tokens
//   (one set for the first global frame, one for the rest, or a single set)
//   followed by source rows, optionally adding a positional table [P, C].
#include "host.hpp"

namespace qv {
namespace {

__global__ void patchify_kernel(const __half* __restrict__ img, __half* __restrict__ out, int S, int H, int W, int p,
                                int kpad, float m0, float m1, float m2, float s0, float s1, float s2) {
  pdl_wait();
  pdl_trigger();
  const int gw = W / p, gh = H / p;
  const long long row = blockIdx.x;   // patch index over S * gh * gw
  const int f = (int)(row / (gh * gw));
  const int pi = (int)(row % (gh * gw));
  const int py = pi / gw, px = pi % gw;
  const __half mean_h[3] = {__float2half_rn(m0), __float2half_rn(m1), __float2half_rn(m2)};
  const __half std_h[3] = {__float2half_rn(s0), __float2half_rn(s1), __float2half_rn(s2)};
  for (int k = threadIdx.x; k < kpad; k += blockDim.x) {
    float v = 0.f;
    if (k < 3 * p * p) {
      const int c = k / (p * p), r = k % (p * p);
      const int ky = r / p, kx = r % p;
      const float x = __half2float(img[(((long long)f * 3 + c) * H + py * p + ky) * W + px * p + kx]);
      const float d = round_f16(x - __half2float(mean_h[c]));
      v = d / __half2float(std_h[c]);
    }
    out[row * kpad + k] = __float2half_rn(v);
  }
}

__global__ void assemble_kernel(const __half* __restrict__ src, long long src_rows_per_frame, long long src_row_off,
                                const __half* __restrict__ specials, int n_special, int two_sets,
                                const __half* __restrict__ pos, __half* __restrict__ out, int P, int C,
                                long long frame_offset) {
  pdl_wait();
  pdl_trigger();
  const long long row = blockIdx.x;  // over S * P
  const long long f = row / P;
  const int p = (int)(row % P);
  const __half* s;
  if (p < n_special) {
    const int set = (two_sets && (f + frame_offset) > 0) ? 1 : 0;
    s = specials + ((long long)set * n_special + p) * C;
  } else {
    s = src + (f * src_rows_per_frame + src_row_off + (p - n_special)) * C;
  }
  for (int c = threadIdx.x * 8; c < C; c += blockDim.x * 8) {
    uint4 u = *reinterpret_cast<const uint4*>(s + c);
    if (pos) {
      uint4 pu = *reinterpret_cast<const uint4*>(pos + (long long)p * C + c);
      uint32_t* a = reinterpret_cast<uint32_t*>(&u);
      const uint32_t* b = reinterpret_cast<const uint32_t*>(&pu);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 x = unpack_half2(a[e]), y = unpack_half2(b[e]);
        a[e] = pack_half2(x.x + y.x, x.y + y.y);
      }
    }
    *reinterpret_cast<uint4*>(out + row * C + c) = u;
  }
}

}  // namespace
}  // namespace qv

using namespace qv;

extern "C" {

int qvggt_patchify(const void* images, void* out, int64_t S, int32_t H, int32_t W, int32_t patch, int32_t k_pad,
                   const float* mean3, const float* std3, void* stream) {
  if (S < 0 || H <= 0 || W <= 0 || patch <= 0 || H % patch || W % patch || k_pad < 3 * patch * patch)
    return set_error(QVGGT_ERR_INVALID, "patchify: bad shape");
  if (!mean3 || !std3) return set_error(QVGGT_ERR_INVALID, "patchify: mean/std required");
  const long long rows = S * (long long)(H / patch) * (W / patch);
  if (rows == 0) return QVGGT_OK;
  if (rows > 2147483647LL) return set_error(QVGGT_ERR_UNSUPPORTED, "patchify: too many patches");
  int rc = check_cuda(launch_pdl(patchify_kernel, dim3((unsigned)rows), dim3(128), 0, static_cast<cudaStream_t>(stream),
                                 1u, static_cast<const __half*>(images), static_cast<__half*>(out), (int)S, (int)H,
                                 (int)W, (int)patch, (int)k_pad, mean3[0], mean3[1], mean3[2], std3[0], std3[1],
                                 std3[2]),
                      "patchify launch");
  if (!rc) count_launch(1);
  return rc;
}

int qvggt_assemble_tokens(const void* src, int64_t src_rows_per_frame, int64_t src_row_offset, const void* specials,
                          int32_t n_special, int32_t two_sets, const void* pos, void* out, int64_t S, int32_t P,
                          int32_t C, int64_t frame_offset, void* stream) {
  if (S < 0 || P <= 0 || C <= 0 || C % 8 || n_special < 0 || n_special > P)
    return set_error(QVGGT_ERR_INVALID, "assemble_tokens: bad shape");
  if (!aligned16(src) || !aligned16(out) || (specials && !aligned16(specials)) || (pos && !aligned16(pos)))
    return set_error(QVGGT_ERR_ALIGN, "assemble_tokens: tensors must be 16-byte aligned");
  if (n_special > 0 && !specials) return set_error(QVGGT_ERR_INVALID, "assemble_tokens: specials required");
  const long long rows = S * (long long)P;
  if (rows == 0) return QVGGT_OK;
  int rc = check_cuda(launch_pdl(assemble_kernel, dim3((unsigned)rows), dim3(128), 0, static_cast<cudaStream_t>(stream),
                                 1u, static_cast<const __half*>(src), (long long)src_rows_per_frame,
                                 (long long)src_row_offset, static_cast<const __half*>(specials), (int)n_special,
                                 (int)two_sets, static_cast<const __half*>(pos), static_cast<__half*>(out), (int)P,
                                 (int)C, (long long)frame_offset),
                      "assemble_tokens launch");
  if (!rc) count_launch(1);
  return rc;
}

}  // extern "C"
