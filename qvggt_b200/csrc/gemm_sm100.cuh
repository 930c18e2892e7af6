// Internal launch description of the tcgen05 GEMM (see gemm_sm100.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace qv {

// B_W4BF: B_W4 with bf16 activations, scales, scaled zeros, bias and output
// (the reference's bf16 instantiation of the same kernels); EPI_STORE only.
enum GemmMode { B_W4 = 0, B_F16 = 1, B_I8 = 2, B_W4BF = 3 };
__host__ __device__ constexpr bool mode_is_w4(int mode) { return mode == B_W4 || mode == B_W4BF; }
enum GemmEpi { EPI_STORE = 0, EPI_GELU = 1, EPI_RESID = 2, EPI_I32 = 3, EPI_QKV_ROPE = 4 };

// EPI_QKV_ROPE: the output columns are [q | k | v] (each `dim` wide, heads of
// 64); q and k get (optional per-head LayerNorm and) VGGT 2-D RoPE, q goes to
// q_out [M, dim], k and v to kv_out [M, 2*dim].
struct RopeEpi {
  void* q_out = nullptr;
  void* kv_out = nullptr;
  int dim = 1024;
  const void* cos_tab = nullptr;   // fp16 [max_pos, 32]
  const void* sin_tab = nullptr;
  int max_pos = 0;
  int tokens_per_frame = 1374, patch_start = 5, grid_w = 37;
  long long token_offset = 0;
  const void* qn_w = nullptr;      // fp16 [64] each, all null = no qk-norm
  const void* qn_b = nullptr;
  const void* kn_w = nullptr;
  const void* kn_b = nullptr;
  float eps = 1e-6f;
};

struct GemmLaunch {
  int mode = B_W4;
  int epi = EPI_STORE;
  const void* a = nullptr;   // [M, lda] fp16 (or int8 for B_I8)
  long long lda = 0;         // elements
  const void* b = nullptr;   // B_W4: qweight int16 [N/4, K]; B_F16: fp16 [N, K]; B_I8: int8 [N, K]
  const void* scales = nullptr;  // B_W4: fp16 [gpad, N]
  const void* zeros = nullptr;   // B_W4: fp16 [gpad, N] (scaled zeros)
  long long gpad = 0;
  int group_size = 128;
  const void* bias = nullptr;    // fp16 [N] or null
  void* out = nullptr;           // fp16 [M, ldo] (int32 for EPI_I32)
  long long ldo = 0;
  const void* resid = nullptr;   // EPI_RESID: fp16 [M, ldr] (may alias out)
  long long ldr = 0;
  const void* gamma = nullptr;   // EPI_RESID: fp16 [N] LayerScale
  const void* wscale = nullptr;  // B_I8: fp16 [N]
  const void* ascale = nullptr;  // B_I8: fp16 [M]
  long long M = 0, N = 0, K = 0;
  RopeEpi rope;                  // EPI_QKV_ROPE only
  bool force_bn128 = false;
  cudaStream_t stream = nullptr;
};

int gemm_launch(const GemmLaunch& L);

// Kernel configurations of gemm_launch (its choice, or a tuning override).
enum GemmConfig { GEMM_CFG_AUTO = 0, GEMM_CFG_PAIR = 1, GEMM_CFG_1SM_256 = 2, GEMM_CFG_1SM_128 = 3 };
int gemm_config_override();   // GEMM_CFG_AUTO unless qvggt_set_gemm_config / QVGGT_GEMM_CONFIG say otherwise
int choose_gemm_config(int mode, long long M, long long N, int sms, bool can_pair, bool can256);
// 2-SM (CTA-pair) variant for large M; called by gemm_launch after validation.
int gemm_launch_2sm(const GemmLaunch& L);

// Small-M split-K GEMM on thread-block clusters (gemm_small.cu): 1 <= M <= 256,
// modes B_W4 / B_F16, epilogues EPI_STORE / EPI_GELU / EPI_RESID.
struct SmallPlan {
  int mt = 16;              // padded row count (the MMA's N)
  int n_blocks = 0;         // 128-channel tiles
  int num_kb = 0;           // 64-wide k-blocks
  int splits = 1;           // K ranges per channel tile = CTAs per cluster (<= 8)
  int kb_per_split = 0;
  int smem = 0;
  int active_clusters = 0;  // co-resident clusters of `splits` CTAs (occupancy query)
};
// Chooses the tile height and K split for the current device; max_splits > 0
// caps the split count.
int gemm_small_plan(int mode, long long M, long long N, long long K, int max_splits, SmallPlan* P);
int gemm_small_launch(const GemmLaunch& L, const SmallPlan& P);

}  // namespace qv
