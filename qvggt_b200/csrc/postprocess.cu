// Camera / geometry post-processing of the heads' outputs (QVGGT's
// qvggt/common/pose_enc.py and geometry.py, which run in PyTorch / numpy on
// the host after the model):
//
// pose_kernel: pose encoding "absT_quaR_FoV" [n, 9] = (t, quaternion x y z w,
//   fov_h, fov_w) -> extrinsics [n, 3, 4] = [R | t] and intrinsics [n, 3, 3]
//   (focal lengths from the fields of view, principal point at the image
//   centre).  One thread per camera.
// unproject_kernel: depth maps [S, H, W] + per-frame extrinsics / intrinsics
//   -> world points [S, H, W, 3] = R^T (cam - t), cam = ((u - cu) d / fu,
//   (v - cv) d / fv, d).  HBM-bound (4 bytes read, 12 written per pixel): each
//   thread takes 4 consecutive pixels with one 16-byte depth load and three
//   16-byte stores, so a warp writes 1.5 KB contiguous; the frame's camera is
//   re-read per pixel group through L1.
#include "host.hpp"

namespace qv {
namespace {

__global__ void pose_kernel(const float* __restrict__ pe, long long n, float h, float w, float* __restrict__ ext,
                            float* __restrict__ intr) {
  pdl_wait();
  pdl_trigger();
  const long long f = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (f >= n) return;
  const float* p = pe + f * 9;
  const float i = p[3], j = p[4], k = p[5], r = p[6];
  const float two_s = 2.f / (i * i + j * j + k * k + r * r);
  float* E = ext + f * 12;
  E[0] = 1.f - two_s * (j * j + k * k);
  E[1] = two_s * (i * j - k * r);
  E[2] = two_s * (i * k + j * r);
  E[3] = p[0];
  E[4] = two_s * (i * j + k * r);
  E[5] = 1.f - two_s * (i * i + k * k);
  E[6] = two_s * (j * k - i * r);
  E[7] = p[1];
  E[8] = two_s * (i * k - j * r);
  E[9] = two_s * (j * k + i * r);
  E[10] = 1.f - two_s * (i * i + j * j);
  E[11] = p[2];
  if (intr) {
    const float pi = 3.14159265358979f;
    const float fov_h = fminf(fmaxf(p[7], 1e-6f), pi - 1e-6f);
    const float fov_w = fminf(fmaxf(p[8], 1e-6f), pi - 1e-6f);
    const float fy = fminf(fmaxf((h * 0.5f) / tanf(fov_h * 0.5f), 1.f), 1e6f);
    const float fx = fminf(fmaxf((w * 0.5f) / tanf(fov_w * 0.5f), 1.f), 1e6f);
    float* K = intr + f * 9;
    K[0] = fx;
    K[1] = 0.f;
    K[2] = w * 0.5f;
    K[3] = 0.f;
    K[4] = fy;
    K[5] = h * 0.5f;
    K[6] = 0.f;
    K[7] = 0.f;
    K[8] = 1.f;
  }
}

__device__ __forceinline__ float3 unproject_one(long long idx, float d, int H, int W, const float* __restrict__ ext,
                                                const float* __restrict__ intr) {
  const long long hw = (long long)H * W;
  const long long s = idx / hw;
  const int pix = (int)(idx - s * hw);
  const int v = pix / W, u = pix - v * W;
  const float* E = ext + s * 12;
  const float* K = intr + s * 9;
  const float fu = fmaxf(__ldg(K + 0), 1e-6f), fv = fmaxf(__ldg(K + 4), 1e-6f);
  const float x = ((float)u - __ldg(K + 2)) * d / fu;
  const float y = ((float)v - __ldg(K + 5)) * d / fv;
  const float r00 = __ldg(E + 0), r01 = __ldg(E + 1), r02 = __ldg(E + 2), t0 = __ldg(E + 3);
  const float r10 = __ldg(E + 4), r11 = __ldg(E + 5), r12 = __ldg(E + 6), t1 = __ldg(E + 7);
  const float r20 = __ldg(E + 8), r21 = __ldg(E + 9), r22 = __ldg(E + 10), t2 = __ldg(E + 11);
  // world = R^T cam + (-R^T t)
  const float w0 = -(r00 * t0 + r10 * t1 + r20 * t2);
  const float w1 = -(r01 * t0 + r11 * t1 + r21 * t2);
  const float w2 = -(r02 * t0 + r12 * t1 + r22 * t2);
  return make_float3(r00 * x + r10 * y + r20 * d + w0, r01 * x + r11 * y + r21 * d + w1,
                     r02 * x + r12 * y + r22 * d + w2);
}

__global__ void unproject_kernel(const float* __restrict__ depth, long long total, int H, int W,
                                 const float* __restrict__ ext, const float* __restrict__ intr,
                                 float* __restrict__ pts) {
  pdl_wait();
  pdl_trigger();
  const long long groups = total / 4;
  for (long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x; g < groups;
       g += (long long)gridDim.x * blockDim.x) {
    const float4 d = __ldg(reinterpret_cast<const float4*>(depth) + g);
    const float3 a = unproject_one(4 * g + 0, d.x, H, W, ext, intr);
    const float3 b = unproject_one(4 * g + 1, d.y, H, W, ext, intr);
    const float3 c = unproject_one(4 * g + 2, d.z, H, W, ext, intr);
    const float3 e = unproject_one(4 * g + 3, d.w, H, W, ext, intr);
    float4* o = reinterpret_cast<float4*>(pts) + 3 * g;
    o[0] = make_float4(a.x, a.y, a.z, b.x);
    o[1] = make_float4(b.y, b.z, c.x, c.y);
    o[2] = make_float4(c.z, e.x, e.y, e.z);
  }
  // the last total % 4 pixels
  const long long tail0 = groups * 4;
  const long long t = tail0 + (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (t < total && t - tail0 < 4) {
    const float3 a = unproject_one(t, __ldg(depth + t), H, W, ext, intr);
    pts[3 * t + 0] = a.x;
    pts[3 * t + 1] = a.y;
    pts[3 * t + 2] = a.z;
  }
}

}  // namespace
}  // namespace qv

using namespace qv;

extern "C" {

int qvggt_pose_encoding_to_extri_intri(const float* pose_enc, int64_t n, int32_t image_h, int32_t image_w,
                                        float* extrinsics, float* intrinsics, void* stream) {
  if (n < 0) return set_error(QVGGT_ERR_INVALID, "pose_encoding_to_extri_intri: n < 0");
  if (intrinsics && (image_h <= 0 || image_w <= 0))
    return set_error(QVGGT_ERR_INVALID, "pose_encoding_to_extri_intri: intrinsics need a positive image size");
  if (n == 0) return QVGGT_OK;
  if (!pose_enc || !extrinsics) return set_error(QVGGT_ERR_INVALID, "pose_encoding_to_extri_intri: null tensor");
  const long long blocks = (n + 127) / 128;
  if (blocks > 2147483647LL) return set_error(QVGGT_ERR_UNSUPPORTED, "pose_encoding_to_extri_intri: n too large");
  int rc = check_cuda(launch_pdl(pose_kernel, dim3((unsigned)blocks), dim3(128), 0, static_cast<cudaStream_t>(stream), 1u,
                                 pose_enc, (long long)n, (float)image_h, (float)image_w, extrinsics, intrinsics),
                      "pose_encoding_to_extri_intri launch");
  if (!rc) count_launch(1);
  return rc;
}

int qvggt_unproject_depth(const float* depth, int64_t S, int32_t H, int32_t W, const float* extrinsics,
                          const float* intrinsics, float* world_points, void* stream) {
  if (S < 0 || H <= 0 || W <= 0) return set_error(QVGGT_ERR_INVALID, "unproject_depth: bad shape");
  const long long total = S * (long long)H * W;
  if (total == 0) return QVGGT_OK;
  if (!depth || !extrinsics || !intrinsics || !world_points)
    return set_error(QVGGT_ERR_INVALID, "unproject_depth: null tensor");
  if (!aligned16(depth) || !aligned16(world_points))
    return set_error(QVGGT_ERR_ALIGN, "unproject_depth: depth and world_points must be 16-byte aligned");
  const DeviceInfo& di = device_info();
  long long blocks = (total / 4 + 255) / 256;
  const long long cap = 8LL * di.num_sms;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  int rc = check_cuda(launch_pdl(unproject_kernel, dim3((unsigned)blocks), dim3(256), 0,
                                 static_cast<cudaStream_t>(stream), 1u, depth, total, (int)H, (int)W, extrinsics,
                                 intrinsics, world_points),
                      "unproject_depth launch");
  if (!rc) count_launch(1);
  return rc;
}

}  // extern "C"
