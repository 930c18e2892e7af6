// Attention for short sequences with head_dim 128 (the camera-head trunk of
// VGGT: 16 heads x 128 over the S camera tokens of each batch, S <= 256):
// softmax(q k^T / sqrt(128)) v, fp16 in / out, fp32 math.
//
// One CTA per (batch, head, chunk of 32 query rows); 8 warps, 4 query rows
// each.  K and V of the (batch, head) are staged in shared memory with a row
// stride of 65 words, so lane j reading key row j (QK^T) or all lanes reading
// one value row (PV) are free of bank conflicts.  QK^T: one lane per key,
// 64 half2 products accumulated in fp32; row max and sum by warp shuffles;
// P goes through a per-warp shared buffer so that each lane accumulates 4 of
// the 128 output dims over all keys.  The work is tiny (S^2 * 128 * 4 FLOP per
// head), so CUDA cores are the right unit; the GEMM-shaped work of the trunk
// runs in the tcgen05 small-M linears.
#include "host.hpp"

namespace qv {
namespace {

constexpr int SA_D = 128;          // head dim
constexpr int SA_MAXL = 256;       // keys per batch
constexpr int SA_ROW = 65;         // shared-memory row stride in 32-bit words (64 half2 + 1)
constexpr int SA_WARPS = 8;
constexpr int SA_QROWS = 32;       // query rows per CTA

struct SmallAttnArgs {
  const __half* q;
  long long q_stride;
  const __half* k;
  const __half* v;
  long long kv_stride;
  __half* out;
  long long o_stride;
  int L, heads, chunks;
  float scale;
};

__global__ void __launch_bounds__(SA_WARPS * 32) attn_small_kernel(SmallAttnArgs a) {
  extern __shared__ uint32_t sm[];
  uint32_t* ks = sm;                                   // [L][SA_ROW] half2 words
  uint32_t* vs = ks + SA_MAXL * SA_ROW;                // [L][SA_ROW]
  float* ps = reinterpret_cast<float*>(vs + SA_MAXL * SA_ROW);   // [SA_WARPS][L]
  uint32_t* qs = reinterpret_cast<uint32_t*>(ps + SA_WARPS * SA_MAXL);   // [SA_WARPS][64]
  pdl_wait();
  pdl_trigger();

  const int chunk = blockIdx.x % a.chunks;
  const int h = (blockIdx.x / a.chunks) % a.heads;
  const int b = blockIdx.x / (a.chunks * a.heads);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int L = a.L;
  const long long row0 = (long long)b * L;

  // stage K and V of this (batch, head): 64 words per row
  for (int idx = threadIdx.x; idx < L * 64; idx += blockDim.x) {
    const int j = idx / 64, w = idx % 64;
    const uint32_t* kp = reinterpret_cast<const uint32_t*>(a.k + (row0 + j) * a.kv_stride + h * SA_D);
    const uint32_t* vp = reinterpret_cast<const uint32_t*>(a.v + (row0 + j) * a.kv_stride + h * SA_D);
    ks[j * SA_ROW + w] = __ldg(kp + w);
    vs[j * SA_ROW + w] = __ldg(vp + w);
  }
  __syncthreads();

  float* p = ps + warp * SA_MAXL;
  uint32_t* qw = qs + warp * 64;
  for (int r = 0; r < SA_QROWS / SA_WARPS; ++r) {
    const int qi = chunk * SA_QROWS + r * SA_WARPS + warp;   // query row within the batch
    if (qi >= L) break;                                      // warp-uniform
    const uint32_t* qp = reinterpret_cast<const uint32_t*>(a.q + (row0 + qi) * a.q_stride + h * SA_D);
    qw[lane] = __ldg(qp + lane);
    qw[lane + 32] = __ldg(qp + lane + 32);
    __syncwarp();
    // scores: lane handles keys lane, lane+32, ...
    float mx = -INFINITY;
    for (int j = lane; j < L; j += 32) {
      float acc = 0.f;
#pragma unroll 16
      for (int w = 0; w < 64; ++w) {
        const float2 qv = unpack_half2(qw[w]);
        const float2 kv = unpack_half2(ks[j * SA_ROW + w]);
        acc = fmaf(qv.x, kv.x, acc);
        acc = fmaf(qv.y, kv.y, acc);
      }
      acc *= a.scale;
      p[j] = acc;
      mx = fmaxf(mx, acc);
    }
    mx = warp_max(mx);
    float sum = 0.f;
    for (int j = lane; j < L; j += 32) {
      const float e = __expf(p[j] - mx);
      p[j] = e;
      sum += e;
    }
    sum = warp_sum(sum);
    __syncwarp();
    // O: lane owns dims 4*lane .. 4*lane+3 (words 2*lane, 2*lane+1)
    float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
    for (int j = 0; j < L; ++j) {
      const float pj = p[j];
      const float2 v01 = unpack_half2(vs[j * SA_ROW + 2 * lane]);
      const float2 v23 = unpack_half2(vs[j * SA_ROW + 2 * lane + 1]);
      o0 = fmaf(pj, v01.x, o0);
      o1 = fmaf(pj, v01.y, o1);
      o2 = fmaf(pj, v23.x, o2);
      o3 = fmaf(pj, v23.y, o3);
    }
    const float inv = 1.f / sum;
    uint2* dst = reinterpret_cast<uint2*>(a.out + (row0 + qi) * a.o_stride + h * SA_D + 4 * lane);
    *dst = make_uint2(pack_half2(o0 * inv, o1 * inv), pack_half2(o2 * inv, o3 * inv));
    __syncwarp();
  }
}

}  // namespace
}  // namespace qv

using namespace qv;

extern "C" int qvggt_attention_small(const void* q, int64_t q_stride, const void* kv, int64_t kv_stride, int64_t k_col0,
                                     int64_t v_col0, void* out, int64_t o_stride, int64_t batches, int64_t L,
                                     int32_t heads, void* stream) {
  if (batches < 0 || L < 0 || heads <= 0) return set_error(QVGGT_ERR_INVALID, "attention_small: bad shape");
  if (L > SA_MAXL) return set_error(QVGGT_ERR_UNSUPPORTED, "attention_small: L=%lld > %d", (long long)L, SA_MAXL);
  if (q_stride % 8 || kv_stride % 8 || o_stride % 8 || k_col0 % 8 || v_col0 % 8)
    return set_error(QVGGT_ERR_ALIGN, "attention_small: strides and column offsets must be multiples of 8");
  if (!aligned16(q) || !aligned16(kv) || !aligned16(out))
    return set_error(QVGGT_ERR_ALIGN, "attention_small: tensors must be 16-byte aligned");
  if (q_stride < heads * SA_D || o_stride < heads * SA_D || kv_stride < k_col0 + heads * SA_D ||
      kv_stride < v_col0 + heads * SA_D)
    return set_error(QVGGT_ERR_INVALID, "attention_small: strides too small for the heads");
  if (batches == 0 || L == 0) return QVGGT_OK;
  SmallAttnArgs a;
  a.q = static_cast<const __half*>(q);
  a.q_stride = q_stride;
  a.k = static_cast<const __half*>(kv) + k_col0;
  a.v = static_cast<const __half*>(kv) + v_col0;
  a.kv_stride = kv_stride;
  a.out = static_cast<__half*>(out);
  a.o_stride = o_stride;
  a.L = (int)L;
  a.heads = heads;
  a.chunks = (int)((L + SA_QROWS - 1) / SA_QROWS);
  a.scale = 0.08838834764831845f;   // 1 / sqrt(128)
  const long long grid = batches * heads * a.chunks;
  if (grid > 2147483647LL) return set_error(QVGGT_ERR_UNSUPPORTED, "attention_small: grid too large");
  const int smem = (2 * SA_MAXL * SA_ROW + SA_WARPS * 64) * 4 + SA_WARPS * SA_MAXL * 4;
  static DeviceFlags attr_set;
  if (int rc = ensure_smem(attr_set, attn_small_kernel, smem, "cudaFuncSetAttribute(attention_small)")) return rc;
  int rc = check_cuda(launch_pdl(attn_small_kernel, dim3((unsigned)grid), dim3(SA_WARPS * 32), smem,
                                 static_cast<cudaStream_t>(stream), 1u, a),
                      "attention_small launch");
  if (!rc) count_launch(1);
  return rc;
}
