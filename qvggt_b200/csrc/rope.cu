// Rotary position embeddings.
//
// rope_with_pos_kernel: the reference's rotate-half RoPE with an explicit fp32
// angle table per (b, s) (fused_rope_with_pos.cu:19-71), any input / output
// strides; one CTA per (s, b), threads over (d2, heads).
//
// qkv_rope2d_kernel: VGGT's 2-D RoPE fused with the q / k / v split of the qkv
// projection.  One thread per (token, head, q|k|v); each thread owns one
// 64-dim head vector (8 x 16-byte loads / stores), applies the optional per-head
// LayerNorm (qk-norm) and the two 1-D rotations (dims 0..31 by the patch row,
// 32..63 by the patch column; rotate-half pairs i <-> i+16 inside each half)
// with the fp16 rounding points of the eager model: h(h(x*cos) + h(rot*sin)).
#include "host.hpp"

namespace qv {
namespace {

__global__ void rope_with_pos_kernel(const __half* __restrict__ in, const float* __restrict__ freqs,
                                     __half* __restrict__ out, int S, int h, int d, int d2, long long is_s,
                                     long long is_b, long long is_h, long long is_d, long long os_s, long long os_b,
                                     long long os_h, long long os_d) {
  pdl_wait();
  pdl_trigger();
  const int s_id = blockIdx.x, b_id = blockIdx.y;
  const __half* src = in + s_id * is_s + b_id * is_b;
  __half* dst = out + s_id * os_s + b_id * os_b;
  const float* f = freqs + ((long long)b_id * S + s_id) * d2;
  const int half_d2 = d2 / 2;
  for (int i = threadIdx.x; i < d2; i += blockDim.x) {
    float sn, cs;
    sincosf(f[i], &sn, &cs);
    for (int hh = threadIdx.y; hh < h; hh += blockDim.y) {
      const __half* sp = src + hh * is_h;
      const float v = __half2float(sp[i * is_d]);
      const float r = (i < half_d2) ? -__half2float(sp[(i + half_d2) * is_d]) : __half2float(sp[(i - half_d2) * is_d]);
      dst[hh * os_h + i * os_d] = __float2half_rn(v * cs + r * sn);
    }
  }
  for (int hh = threadIdx.y; hh < h; hh += blockDim.y)
    for (int i = d2 + threadIdx.x; i < d; i += blockDim.x) dst[hh * os_h + i * os_d] = src[hh * is_h + i * is_d];
}

struct Rope2dArgs {
  const __half* qkv;
  __half* q_out;
  __half* kv_out;
  long long T;
  int heads;
  long long token_offset;
  int tokens_per_frame, patch_start, grid_w, max_pos;
  const __half* cos_tab;
  const __half* sin_tab;
  int qk_norm;
  const __half *qn_w, *qn_b, *kn_w, *kn_b;
  float eps;
};

__device__ __forceinline__ void head_layernorm(float (&v)[64], const __half* w, const __half* b, float eps) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 64; ++i) s += v[i];
  const float mean = s * (1.f / 64.f);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < 64; ++i) q = fmaf(v[i] - mean, v[i] - mean, q);
  const float rstd = rsqrtf(q * (1.f / 64.f) + eps);
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = round_f16(fmaf((v[i] - mean) * rstd, __half2float(w[i]), __half2float(b[i])));
}

// One 32-dim half rotated by position p (tables are [max_pos, 32]).
__device__ __forceinline__ void rope_half(const float* x, float* y, const __half* cos_row, const __half* sin_row) {
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float c = __half2float(cos_row[i]);
    const float s = __half2float(sin_row[i]);
    const float r = (i < 16) ? -x[i + 16] : x[i - 16];
    y[i] = round_f16(round_f16(x[i] * c) + round_f16(r * s));
  }
}

__global__ void __launch_bounds__(128) qkv_rope2d_kernel(Rope2dArgs a) {
  pdl_wait();
  pdl_trigger();
  const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int per_tok = 3 * a.heads;
  const long long t = gid / per_tok;
  if (t >= a.T) return;
  const int r = (int)(gid % per_tok);
  const int which = r / a.heads;  // 0 = q, 1 = k, 2 = v
  const int hh = r % a.heads;
  const int C = a.heads * 64;
  const uint4* src = reinterpret_cast<const uint4*>(a.qkv + t * 3 * C + which * C + hh * 64);
  uint4* dst = (which == 0) ? reinterpret_cast<uint4*>(a.q_out + t * C + hh * 64)
                            : reinterpret_cast<uint4*>(a.kv_out + t * 2 * C + (which - 1) * C + hh * 64);
  if (which == 2) {
#pragma unroll
    for (int j = 0; j < 8; ++j) dst[j] = src[j];
    return;
  }
  float v[64];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    uint4 u = src[j];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float2 f = unpack_half2(w[e]);
      v[8 * j + 2 * e] = f.x;
      v[8 * j + 2 * e + 1] = f.y;
    }
  }
  if (a.qk_norm) {
    if (which == 0) head_layernorm(v, a.qn_w, a.qn_b, a.eps);
    else head_layernorm(v, a.kn_w, a.kn_b, a.eps);
  }
  const int p = (int)((t + a.token_offset) % a.tokens_per_frame);
  int py = 0, px = 0;
  if (p >= a.patch_start) {
    const int q = p - a.patch_start;
    py = q / a.grid_w + 1;
    px = q % a.grid_w + 1;
  }
  py = min(py, a.max_pos - 1);
  px = min(px, a.max_pos - 1);
  float y[64];
  rope_half(v, y, a.cos_tab + py * 32, a.sin_tab + py * 32);
  rope_half(v + 32, y + 32, a.cos_tab + px * 32, a.sin_tab + px * 32);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] = pack_half2(y[8 * j + 2 * e], y[8 * j + 2 * e + 1]);
    dst[j] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace
}  // namespace qv

using namespace qv;

extern "C" {

int qvggt_rope_with_pos(const void* in, const float* freqs, void* out, int64_t s, int64_t b, int64_t h, int64_t d,
                        int64_t d2, const int64_t* in_strides, const int64_t* out_strides, void* stream) {
  if (s < 0 || b < 0 || h <= 0 || d <= 0 || d2 < 0 || d2 > d || d2 % 2)
    return set_error(QVGGT_ERR_INVALID, "rope_with_pos: bad shape");
  if (!in_strides || !out_strides) return set_error(QVGGT_ERR_INVALID, "rope_with_pos: strides required");
  if (s == 0 || b == 0) return QVGGT_OK;
  if (s > 2147483647 || b > 65535) return set_error(QVGGT_ERR_UNSUPPORTED, "rope_with_pos: grid too large");
  const int warps = h < 16 ? 4 : 8;  // launch shape as fused_rope_with_pos.cu:80-82
  int rc = check_cuda(
      launch_pdl(rope_with_pos_kernel, dim3((unsigned)s, (unsigned)b), dim3(32, warps), 0,
                 static_cast<cudaStream_t>(stream), 1u, static_cast<const __half*>(in), freqs, static_cast<__half*>(out),
                 (int)s, (int)h, (int)d, (int)d2, (long long)in_strides[0], (long long)in_strides[1],
                 (long long)in_strides[2], (long long)in_strides[3], (long long)out_strides[0],
                 (long long)out_strides[1], (long long)out_strides[2], (long long)out_strides[3]),
      "rope_with_pos launch");
  if (!rc) count_launch(1);
  return rc;
}

int qvggt_qkv_rope2d(const void* qkv, void* q_out, void* kv_out, int64_t T, int32_t heads, int64_t token_offset,
                     int32_t tokens_per_frame, int32_t patch_start, int32_t grid_w, const void* cos_tab,
                     const void* sin_tab, int32_t max_pos, int32_t qk_norm, const void* qn_w, const void* qn_b,
                     const void* kn_w, const void* kn_b, float eps, void* stream) {
  if (T < 0 || heads <= 0 || tokens_per_frame <= 0 || grid_w <= 0 || max_pos <= 0 || patch_start < 0)
    return set_error(QVGGT_ERR_INVALID, "qkv_rope2d: bad arguments");
  if (!aligned16(qkv) || !aligned16(q_out) || !aligned16(kv_out))
    return set_error(QVGGT_ERR_ALIGN, "qkv_rope2d: tensors must be 16-byte aligned");
  if (qk_norm && (!qn_w || !qn_b || !kn_w || !kn_b))
    return set_error(QVGGT_ERR_INVALID, "qkv_rope2d: qk_norm needs weights");
  if (T == 0) return QVGGT_OK;
  Rope2dArgs a;
  a.qkv = static_cast<const __half*>(qkv);
  a.q_out = static_cast<__half*>(q_out);
  a.kv_out = static_cast<__half*>(kv_out);
  a.T = T;
  a.heads = heads;
  a.token_offset = token_offset;
  a.tokens_per_frame = tokens_per_frame;
  a.patch_start = patch_start;
  a.grid_w = grid_w;
  a.max_pos = max_pos;
  a.cos_tab = static_cast<const __half*>(cos_tab);
  a.sin_tab = static_cast<const __half*>(sin_tab);
  a.qk_norm = qk_norm;
  a.qn_w = static_cast<const __half*>(qn_w);
  a.qn_b = static_cast<const __half*>(qn_b);
  a.kn_w = static_cast<const __half*>(kn_w);
  a.kn_b = static_cast<const __half*>(kn_b);
  a.eps = eps;
  const long long threads = T * 3 * heads;
  const unsigned blocks = (unsigned)((threads + 127) / 128);
  int rc = check_cuda(launch_pdl(qkv_rope2d_kernel, dim3(blocks), dim3(128), 0, static_cast<cudaStream_t>(stream), 1u, a),
                      "qkv_rope2d launch");
  if (!rc) count_launch(1);
  return rc;
}

}  // extern "C"
