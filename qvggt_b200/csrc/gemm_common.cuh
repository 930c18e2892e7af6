// Shared pieces of the tcgen05 GEMM kernels (1-SM and 2-SM variants): the
// argument block, the fused epilogues and the bit-exact int4 dequantisation.
#pragma once

#include "common.cuh"
#include "gemm_sm100.cuh"

namespace qv {
namespace gemmk {

struct GemmArgs {
  int M, N, K;
  int n_blocks, num_tiles, num_kb;
  int group_size;
  int epi;
  const __half* bias;
  __half* out;
  long long ldo;
  const __half* resid;
  long long ldr;
  const __half* gamma;
  const __half* wscale;
  const __half* ascale;
  RopeEpi rope;
  Ctl ctl;
};

// EPI_QKV_ROPE for one 64-wide head of one row: y = half(half(acc) + bias),
// then for q / k heads the optional per-head LayerNorm and the 2-D RoPE of the
// VGGT aggregator (dims 0..31 rotated by the patch row, 32..63 by the patch
// column, rotate-half pairs i <-> i+16, h(h(x*cos) + h(rot*sin))), stored to
// q_out or kv_out.  Every intermediate y is an fp16 value, so the head is held
// as 32 packed half2 words (yh[k] = y[2k], y[2k+1]): the arithmetic is the
// same fp32 sequence, at half the registers (the W4 GEMM runs 512 threads
// with 128 registers each).
__device__ __forceinline__ void epilogue_qkv_head(const GemmArgs& g, int row, int col0, const uint32_t (&r)[64]) {
  const RopeEpi& R = g.rope;
  const int region = col0 / R.dim;           // 0 = q, 1 = k, 2 = v
  const int hcol = col0 - region * R.dim;    // column of the head inside its region
  uint32_t yh[32];
  const uint4* bp = reinterpret_cast<const uint4*>(g.bias + col0);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    uint4 bu = g.bias ? __ldg(bp + j) : make_uint4(0, 0, 0, 0);
    const uint32_t b4[4] = {bu.x, bu.y, bu.z, bu.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 b = unpack_half2(b4[e]);
      yh[4 * j + e] = pack_half2(round_f16(__uint_as_float(r[8 * j + 2 * e])) + b.x,
                                 round_f16(__uint_as_float(r[8 * j + 2 * e + 1])) + b.y);
    }
  }
  __half* dst;
  if (region == 0) {
    dst = reinterpret_cast<__half*>(R.q_out) + (long long)row * R.dim + hcol;
  } else {
    dst = reinterpret_cast<__half*>(R.kv_out) + (long long)row * 2 * R.dim + (region - 1) * R.dim + hcol;
  }
  if (region < 2) {
    const __half* nw = reinterpret_cast<const __half*>(region == 0 ? R.qn_w : R.kn_w);
    const __half* nb = reinterpret_cast<const __half*>(region == 0 ? R.qn_b : R.kn_b);
    if (nw) {
      float s = 0.f;
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        const float2 y = unpack_half2(yh[k]);
        s += y.x;
        s += y.y;
      }
      const float mean = s * (1.f / 64.f);
      float q = 0.f;
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        const float2 y = unpack_half2(yh[k]);
        q = fmaf(y.x - mean, y.x - mean, q);
        q = fmaf(y.y - mean, y.y - mean, q);
      }
      const float rstd = rsqrtf(q * (1.f / 64.f) + R.eps);
      const uint32_t* nw2 = reinterpret_cast<const uint32_t*>(nw);
      const uint32_t* nb2 = reinterpret_cast<const uint32_t*>(nb);
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        const float2 y = unpack_half2(yh[k]);
        const float2 w = unpack_half2(__ldg(nw2 + k)), b = unpack_half2(__ldg(nb2 + k));
        yh[k] = pack_half2(fmaf((y.x - mean) * rstd, w.x, b.x), fmaf((y.y - mean) * rstd, w.y, b.y));
      }
    }
    const int p = (int)(((long long)row + R.token_offset) % R.tokens_per_frame);
    int py = 0, px = 0;
    if (p >= R.patch_start) {
      const int q = p - R.patch_start;
      py = min(q / R.grid_w + 1, R.max_pos - 1);
      px = min(q % R.grid_w + 1, R.max_pos - 1);
    }
    const __half* ct = reinterpret_cast<const __half*>(R.cos_tab);
    const __half* st = reinterpret_cast<const __half*>(R.sin_tab);
    // The tables hold each angle twice (columns i and i+16 are equal), so the
    // pair (i, i+16) shares one cos / sin: rotate it in place.  Columns i and
    // i+1 (i even) are one packed word, as are i+16 and i+17.
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int pp = half ? px : py;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const uint4 cu = __ldg(reinterpret_cast<const uint4*>(ct + pp * 32) + j);
        const uint4 su = __ldg(reinterpret_cast<const uint4*>(st + pp * 32) + j);
        const uint32_t c4[4] = {cu.x, cu.y, cu.z, cu.w}, s4[4] = {su.x, su.y, su.z, su.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int k = 16 * half + 4 * j + e;   // word of columns 2k, 2k+1; its partner is word k+8
          const float2 cs = unpack_half2(c4[e]), sn = unpack_half2(s4[e]);
          const float2 a = unpack_half2(yh[k]), bq = unpack_half2(yh[k + 8]);
          yh[k] = pack_half2(round_f16(a.x * cs.x) + round_f16(-bq.x * sn.x),
                             round_f16(a.y * cs.y) + round_f16(-bq.y * sn.y));
          yh[k + 8] = pack_half2(round_f16(bq.x * cs.x) + round_f16(a.x * sn.x),
                                 round_f16(bq.y * cs.y) + round_f16(a.y * sn.y));
        }
      }
    }
  }
  uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int j = 0; j < 8; ++j) d4[j] = make_uint4(yh[4 * j], yh[4 * j + 1], yh[4 * j + 2], yh[4 * j + 3]);
}

__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }

// Epilogue for 16 consecutive columns of one row held as fp32 (or s32) bits.
template <int MODE>
__device__ __forceinline__ void epilogue16(const GemmArgs& g, int row, int col, const uint32_t (&r)[16]) {
  if constexpr (MODE == B_W4BF) {
    // bf16 store: y = bf16(acc), or bf16(bf16(acc) + bias) (EPI_STORE only)
    uint32_t o[8];
    if (g.bias != nullptr) {
      const uint4* bp = reinterpret_cast<const uint4*>(g.bias + col);
      uint32_t bu[8];
      *reinterpret_cast<uint4*>(&bu[0]) = __ldg(bp);
      *reinterpret_cast<uint4*>(&bu[4]) = __ldg(bp + 1);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float2 b = unpack_bf162(bu[i]);
        o[i] = pack_bf162(round_bf16(__uint_as_float(r[2 * i])) + b.x, round_bf16(__uint_as_float(r[2 * i + 1])) + b.y);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = pack_bf162(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
    }
    uint4* op = reinterpret_cast<uint4*>(g.out + (long long)row * g.ldo + col);
    op[0] = *reinterpret_cast<uint4*>(&o[0]);
    op[1] = *reinterpret_cast<uint4*>(&o[4]);
    return;
  }
  float y[16];
  if constexpr (MODE == B_I8) {
    if (g.epi == EPI_I32) {
      uint4* op = reinterpret_cast<uint4*>(reinterpret_cast<int32_t*>(g.out) + (long long)row * g.ldo + col);
#pragma unroll
      for (int i = 0; i < 4; ++i) op[i] = make_uint4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]);
      return;
    }
    const float as = __half2float(g.ascale[row]);
    const uint4* wsp = reinterpret_cast<const uint4*>(g.wscale + col);
    uint32_t wsu[8];
    *reinterpret_cast<uint4*>(&wsu[0]) = __ldg(wsp);
    *reinterpret_cast<uint4*>(&wsu[4]) = __ldg(wsp + 1);
    if (g.bias != nullptr) {
      const uint4* bp = reinterpret_cast<const uint4*>(g.bias + col);
      uint32_t bu[8];
      *reinterpret_cast<uint4*>(&bu[0]) = __ldg(bp);
      *reinterpret_cast<uint4*>(&bu[4]) = __ldg(bp + 1);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float2 ws = unpack_half2(wsu[i]);
        float2 b = unpack_half2(bu[i]);
        // (acc * ws) * as + bias, contracted (w8a8_gemm_cuda.cu:551-556)
        y[2 * i] = __fmaf_rn(__fmul_rn(__int2float_rn((int)r[2 * i]), ws.x), as, b.x);
        y[2 * i + 1] = __fmaf_rn(__fmul_rn(__int2float_rn((int)r[2 * i + 1]), ws.y), as, b.y);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float2 ws = unpack_half2(wsu[i]);
        // acc * (ws * as) (w8a8_gemm_cuda.cu:868-873)
        y[2 * i] = __fmul_rn(__int2float_rn((int)r[2 * i]), __fmul_rn(ws.x, as));
        y[2 * i + 1] = __fmul_rn(__int2float_rn((int)r[2 * i + 1]), __fmul_rn(ws.y, as));
      }
    }
    if (g.epi == EPI_RESID) {
      // out = resid + half(half(y) * gamma): the W8A8 linear's fp16 output,
      // then the LayerScale residual add of the block
      const uint4* gp = reinterpret_cast<const uint4*>(g.gamma + col);
      const uint4* rp = reinterpret_cast<const uint4*>(g.resid + (long long)row * g.ldr + col);
      uint32_t gu[8], ru[8];
      *reinterpret_cast<uint4*>(&gu[0]) = __ldg(gp);
      *reinterpret_cast<uint4*>(&gu[4]) = __ldg(gp + 1);
      *reinterpret_cast<uint4*>(&ru[0]) = rp[0];
      *reinterpret_cast<uint4*>(&ru[4]) = rp[1];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float2 gm = unpack_half2(gu[i]);
        const float2 x = unpack_half2(ru[i]);
        y[2 * i] = x.x + round_f16(round_f16(y[2 * i]) * gm.x);
        y[2 * i + 1] = x.y + round_f16(round_f16(y[2 * i + 1]) * gm.y);
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) y[i] = round_f16(__uint_as_float(r[i]));
    if (g.bias != nullptr) {
      const uint4* bp = reinterpret_cast<const uint4*>(g.bias + col);
      uint32_t bu[8];
      *reinterpret_cast<uint4*>(&bu[0]) = __ldg(bp);
      *reinterpret_cast<uint4*>(&bu[4]) = __ldg(bp + 1);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float2 b = unpack_half2(bu[i]);
        y[2 * i] = round_f16(y[2 * i] + b.x);
        y[2 * i + 1] = round_f16(y[2 * i + 1] + b.y);
      }
    }
    if (g.epi == EPI_GELU) {
#pragma unroll
      for (int i = 0; i < 16; ++i) y[i] = gelu_erf(y[i]);
    } else if (g.epi == EPI_RESID) {
      const uint4* gp = reinterpret_cast<const uint4*>(g.gamma + col);
      const uint4* rp = reinterpret_cast<const uint4*>(g.resid + (long long)row * g.ldr + col);
      uint32_t gu[8], ru[8];
      *reinterpret_cast<uint4*>(&gu[0]) = __ldg(gp);
      *reinterpret_cast<uint4*>(&gu[4]) = __ldg(gp + 1);
      *reinterpret_cast<uint4*>(&ru[0]) = rp[0];
      *reinterpret_cast<uint4*>(&ru[4]) = rp[1];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float2 gm = unpack_half2(gu[i]);
        float2 x = unpack_half2(ru[i]);
        y[2 * i] = x.x + round_f16(y[2 * i] * gm.x);
        y[2 * i + 1] = x.y + round_f16(y[2 * i + 1] * gm.y);
      }
    }
  }
  uint32_t o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = pack_half2(y[2 * i], y[2 * i + 1]);
  uint4* op = reinterpret_cast<uint4*>(g.out + (long long)row * g.ldo + col);
  op[0] = *reinterpret_cast<uint4*>(&o[0]);
  op[1] = *reinterpret_cast<uint4*>(&o[4]);
}

// Dequantise one 16-byte chunk (4 u32 = 32 nibbles of one channel, covering
// 32 consecutive k) into four 16-byte fp16 chunks (8 consecutive k each).
//
// Word w of a channel's 16-word segment holds, in nibble j, k = 32*(w/8) + w%8 + 8j
// (relative to its 64-wide k-chunk).  The u32 formed by words (2u, 2u+1)
// therefore holds the k pair (b, b+1), b = 2u (mod 8), in nibbles (j, j+4) for
// each j, i.e. in the 16-bit halves of (x >> 4j) & 0x000F000F.  OR-ing the
// exponent pattern 0x6400 makes each half the fp16 value 1024 + q exactly;
// subtracting 1024 leaves the exact integer q; one fused multiply-add applies
// the group scale and scaled zero (rounded once, as the reference's __hfma2).
// BF = true: the bf16 form (dequantize.cuh:53-90) -- exponent pattern 0x4300
// (bf16 128 + q, exact since the bf16 spacing at 128 is 1), subtract 128, one
// bf16x2 fma.  s2 / z2 hold the scale and scaled zero in both halves.
template <bool BF = false>
__device__ __forceinline__ void dequant_chunk(const uint32_t (&x)[4], uint32_t s2, uint32_t z2, uint4 (&out)[4]) {
  constexpr uint32_t kMagic = BF ? 0x43004300u : 0x64006400u;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t o[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      uint32_t t;
      const uint32_t src = x[u] >> (4 * q);
      asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(t) : "r"(src), "r"(0x000F000Fu), "r"(kMagic));
      if constexpr (BF) {
        using T2 = __nv_bfloat162;
        const uint32_t m = kMagic;
        const T2 w = __hfma2(__hsub2(*reinterpret_cast<const T2*>(&t), *reinterpret_cast<const T2*>(&m)),
                             *reinterpret_cast<const T2*>(&s2), *reinterpret_cast<const T2*>(&z2));
        o[u] = *reinterpret_cast<const uint32_t*>(&w);
      } else {
        using T2 = __half2;
        const uint32_t m = kMagic;
        const T2 w = __hfma2(__hsub2(*reinterpret_cast<const T2*>(&t), *reinterpret_cast<const T2*>(&m)),
                             *reinterpret_cast<const T2*>(&s2), *reinterpret_cast<const T2*>(&z2));
        o[u] = *reinterpret_cast<const uint32_t*>(&w);
      }
    }
    out[q] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}
// Both halves of a 32-bit word set to one 16-bit value (scale / scaled zero).
__device__ __forceinline__ uint32_t dup16(const void* p) {
  const uint32_t v = *reinterpret_cast<const uint16_t*>(p);
  return v | (v << 16);
}


}  // namespace gemmk
}  // namespace qv
