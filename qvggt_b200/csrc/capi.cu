// C ABI: library state (errors, device status word, wait budget, tensor-map
// encoding) and the GEMM entry points.  The other kernels' entry points live
// beside their kernels.
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "gemm_sm100.cuh"
#include "host.hpp"

namespace qv {

namespace {
thread_local char g_errmsg[512] = {0};
std::atomic<unsigned long long> g_timeout_ns{2000000000ull};
std::atomic<uint64_t> g_launches{0};
DeviceInfo g_dev[kMaxDevices];
std::once_flag g_dev_once[kMaxDevices];
uint32_t* g_status_ptr[kMaxDevices] = {};
std::once_flag g_status_once[kMaxDevices];

int current_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}

void query_device(DeviceInfo& d, int dev) {
  cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev);
  d.device = dev;
}
}  // namespace

// The device status word.  One per device (every device that loads the
// library holds its own copy); kernels receive its address in their Ctl.
__device__ uint32_t g_device_status[4];

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_errmsg, sizeof(g_errmsg), fmt, ap);
  va_end(ap);
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return QVGGT_OK;
  return set_error(QVGGT_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

void count_launch(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("QVGGT_PDL");
    return !(e && e[0] == '0' && e[1] == 0);
  }();
  return on;
}

const DeviceInfo& device_info() {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) {   // not cached: queried on every call
    thread_local DeviceInfo d;
    query_device(d, dev);
    return d;
  }
  std::call_once(g_dev_once[dev], [dev] { query_device(g_dev[dev], dev); });
  return g_dev[dev];
}

// Address of the current device's status word (the host-side name of a
// __device__ variable is not a device address: it is looked up once per device
// with that device current).
static uint32_t* status_ptr() {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) {
    void* p = nullptr;
    return cudaGetSymbolAddress(&p, g_device_status) == cudaSuccess ? static_cast<uint32_t*>(p) : nullptr;
  }
  std::call_once(g_status_once[dev], [dev] {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_status) == cudaSuccess) g_status_ptr[dev] = static_cast<uint32_t*>(p);
  });
  return g_status_ptr[dev];
}

Ctl make_ctl() {
  Ctl c;
  c.status = status_ptr();
  c.timeout_ns = g_timeout_ns.load(std::memory_order_relaxed);
  return c;
}

int encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
                const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !p)
      return set_error(QVGGT_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5];
  cuuint32_t es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    es[i] = 1;
    if (i < rank - 1) s[i] = strides_bytes[i];
  }
  CUresult r = fn(map, dtype, (cuuint32_t)rank, const_cast<void*>(base), d, s, b, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(QVGGT_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return QVGGT_OK;
}

// Self-test kernel: one bounded wait on a barrier nothing arrives on.
__global__ void selftest_wait_kernel(Ctl ctl) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(&bar, 0, &abort_flag, ctl, ST_TIMEOUT_SELFTEST);
  __syncthreads();
}

}  // namespace qv

using namespace qv;

extern "C" {

int qvggt_version(void) { return 100; }

const char* qvggt_last_error(void) { return g_errmsg; }

uint64_t qvggt_launch_count(void) { return g_launches.load(); }

int qvggt_set_wait_timeout_ns(uint64_t ns) {
  if (ns == 0) return set_error(QVGGT_ERR_INVALID, "timeout must be > 0");
  g_timeout_ns.store(ns);
  return QVGGT_OK;
}

int qvggt_device_status(uint32_t* status_out, int clear) {
  int rc = check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  if (rc) return rc;
  uint32_t v[4] = {0, 0, 0, 0};
  rc = check_cuda(cudaMemcpyFromSymbol(v, g_device_status, sizeof(v)), "read status");
  if (rc) return rc;
  if (status_out) *status_out = v[0];
  if (clear) {
    uint32_t z[4] = {0, 0, 0, 0};
    rc = check_cuda(cudaMemcpyToSymbol(g_device_status, z, sizeof(z)), "clear status");
    if (rc) return rc;
  }
  return QVGGT_OK;
}

int qvggt_selftest_wait_timeout(uint64_t timeout_ns, uint32_t* status_out) {
  uint32_t st = 0;
  int rc = qvggt_device_status(&st, 1);
  if (rc) return rc;
  Ctl ctl = make_ctl();
  ctl.timeout_ns = timeout_ns;
  selftest_wait_kernel<<<1, 32>>>(ctl);
  count_launch(1);
  rc = check_cuda(cudaGetLastError(), "selftest launch");
  if (rc) return rc;
  rc = qvggt_device_status(&st, 1);
  if (rc) return rc;
  if (status_out) *status_out = st;
  return st == ST_TIMEOUT_SELFTEST ? QVGGT_ERR_TIMEOUT : QVGGT_OK;
}

int qvggt_w4a16_gemm(const void* in_feats, const void* qweight, const void* scales, const void* scaled_zeros,
                     const void* bias, void* out, int64_t M, int64_t N, int64_t K, int64_t gpad,
                     int32_t group_size, void* stream) {
  return qvggt_w4a16_linear_ex(in_feats, K, qweight, scales, scaled_zeros, bias, out, N, M, N, K, gpad, group_size,
                               0, nullptr, 0, nullptr, stream);
}

int qvggt_w4a16_gemm_bf16(const void* in_feats, const void* qweight, const void* scales, const void* scaled_zeros,
                          const void* bias, void* out, int64_t M, int64_t N, int64_t K, int64_t gpad,
                          int32_t group_size, void* stream) {
  GemmLaunch L;
  L.mode = B_W4BF;
  L.epi = EPI_STORE;
  L.a = in_feats; L.lda = K; L.b = qweight; L.scales = scales; L.zeros = scaled_zeros; L.gpad = gpad;
  L.group_size = group_size; L.bias = bias; L.out = out; L.ldo = N;
  L.M = M; L.N = N; L.K = K; L.stream = static_cast<cudaStream_t>(stream);
  int rc = gemm_launch(L);
  if (rc == QVGGT_OK && M > 0) count_launch(1);
  return rc;
}

int qvggt_w4a16_linear_ex(const void* in_feats, int64_t lda, const void* qweight, const void* scales,
                          const void* scaled_zeros, const void* bias, void* out, int64_t ldo, int64_t M, int64_t N,
                          int64_t K, int64_t gpad, int32_t group_size, int32_t act, const void* resid,
                          int64_t ldr, const void* gamma, void* stream) {
  GemmLaunch L;
  L.mode = B_W4;
  L.epi = resid ? EPI_RESID : (act == 1 ? EPI_GELU : EPI_STORE);
  if (resid && act) return set_error(QVGGT_ERR_INVALID, "act and residual are exclusive");
  if (resid && resid != out) return set_error(QVGGT_ERR_INVALID, "residual epilogue updates in place: out == resid");
  if (lda % 8 || ldo % 8 || (resid && ldr % 8)) return set_error(QVGGT_ERR_ALIGN, "strides must be multiples of 8");
  L.a = in_feats; L.lda = lda; L.b = qweight; L.scales = scales; L.zeros = scaled_zeros; L.gpad = gpad;
  L.group_size = group_size; L.bias = bias; L.out = out; L.ldo = ldo; L.resid = resid; L.ldr = ldr;
  L.gamma = gamma; L.M = M; L.N = N; L.K = K; L.stream = static_cast<cudaStream_t>(stream);
  int rc = gemm_launch(L);
  if (rc == QVGGT_OK && M > 0) count_launch(1);
  return rc;
}

int qvggt_qkv_rope_linear(const void* in_feats, int32_t weight_kind, const void* qweight, const void* scales,
                          const void* scaled_zeros, int64_t gpad, int32_t group_size, const void* bias, void* q_out,
                          void* kv_out, int64_t M, int64_t K, int32_t dim, int64_t token_offset,
                          int32_t tokens_per_frame, int32_t patch_start, int32_t grid_w, const void* cos_tab,
                          const void* sin_tab, int32_t max_pos, int32_t qk_norm, const void* qn_w, const void* qn_b,
                          const void* kn_w, const void* kn_b, float eps, void* stream) {
  if (weight_kind != 0 && weight_kind != 1) return set_error(QVGGT_ERR_INVALID, "qkv_rope_linear: weight_kind");
  if (qk_norm && (!qn_w || !qn_b || !kn_w || !kn_b))
    return set_error(QVGGT_ERR_INVALID, "qkv_rope_linear: qk_norm needs weights");
  GemmLaunch L;
  L.mode = weight_kind == 0 ? B_W4 : B_F16;
  L.epi = EPI_QKV_ROPE;
  L.a = in_feats; L.lda = K; L.b = qweight; L.scales = scales; L.zeros = scaled_zeros; L.gpad = gpad;
  L.group_size = group_size; L.bias = bias; L.out = q_out; L.ldo = dim;
  L.M = M; L.N = 3LL * dim; L.K = K; L.stream = static_cast<cudaStream_t>(stream);
  L.rope.q_out = q_out; L.rope.kv_out = kv_out; L.rope.dim = dim; L.rope.cos_tab = cos_tab; L.rope.sin_tab = sin_tab;
  L.rope.max_pos = max_pos; L.rope.tokens_per_frame = tokens_per_frame; L.rope.patch_start = patch_start;
  L.rope.grid_w = grid_w; L.rope.token_offset = token_offset; L.rope.eps = eps;
  if (qk_norm) { L.rope.qn_w = qn_w; L.rope.qn_b = qn_b; L.rope.kn_w = kn_w; L.rope.kn_b = kn_b; }
  int rc = gemm_launch(L);
  if (rc == QVGGT_OK && M > 0) count_launch(1);
  return rc;
}

int qvggt_f16_linear_ex(const void* in_feats, int64_t lda, const void* weight, const void* bias, void* out,
                        int64_t ldo, int64_t M, int64_t N, int64_t K, int32_t act, const void* resid, int64_t ldr,
                        const void* gamma, void* stream) {
  GemmLaunch L;
  L.mode = B_F16;
  L.epi = resid ? EPI_RESID : (act == 1 ? EPI_GELU : EPI_STORE);
  if (resid && act) return set_error(QVGGT_ERR_INVALID, "act and residual are exclusive");
  if (resid && resid != out) return set_error(QVGGT_ERR_INVALID, "residual epilogue updates in place: out == resid");
  if (lda % 8 || ldo % 8 || (resid && ldr % 8)) return set_error(QVGGT_ERR_ALIGN, "strides must be multiples of 8");
  L.a = in_feats; L.lda = lda; L.b = weight; L.bias = bias; L.out = out; L.ldo = ldo; L.resid = resid;
  L.ldr = ldr; L.gamma = gamma; L.M = M; L.N = N; L.K = K; L.stream = static_cast<cudaStream_t>(stream);
  int rc = gemm_launch(L);
  if (rc == QVGGT_OK && M > 0) count_launch(1);
  return rc;
}

// weight_kind of qvggt_small_linear -> GemmMode (-1: invalid)
static int small_mode(int32_t weight_kind) {
  return weight_kind == 0 ? B_W4 : weight_kind == 1 ? B_F16 : weight_kind == 2 ? B_W4BF : -1;
}

int qvggt_small_linear_plan(int32_t weight_kind, int64_t M, int64_t N, int64_t K, int32_t* info) {
  if (!info) return set_error(QVGGT_ERR_INVALID, "small_linear_plan: info is null");
  if (small_mode(weight_kind) < 0) return set_error(QVGGT_ERR_INVALID, "small_linear: weight_kind");
  SmallPlan P;
  int rc = gemm_small_plan(small_mode(weight_kind), M, N, K, 0, &P);
  if (rc) return rc;
  info[0] = P.mt;
  info[1] = P.splits;
  info[2] = P.kb_per_split;
  info[3] = P.n_blocks * P.splits;
  info[4] = P.active_clusters;
  return QVGGT_OK;
}

int qvggt_small_linear(int32_t weight_kind, const void* in_feats, int64_t lda, const void* weight, const void* scales,
                       const void* scaled_zeros, int64_t gpad, int32_t group_size, const void* bias, void* out,
                       int64_t ldo, int64_t M, int64_t N, int64_t K, int32_t act, const void* resid, int64_t ldr,
                       const void* gamma, void* stream) {
  const int mode = small_mode(weight_kind);
  if (mode < 0) return set_error(QVGGT_ERR_INVALID, "small_linear: weight_kind");
  if (resid && act) return set_error(QVGGT_ERR_INVALID, "act and residual are exclusive");
  if (resid && resid != out) return set_error(QVGGT_ERR_INVALID, "residual epilogue updates in place: out == resid");
  SmallPlan P;
  int rc = gemm_small_plan(mode, M, N, K, 0, &P);
  if (rc) return rc;
  GemmLaunch L;
  L.mode = mode;
  L.epi = resid ? EPI_RESID : (act == 1 ? EPI_GELU : EPI_STORE);
  L.a = in_feats; L.lda = lda; L.b = weight; L.scales = scales; L.zeros = scaled_zeros; L.gpad = gpad;
  L.group_size = group_size; L.bias = bias; L.out = out; L.ldo = ldo; L.resid = resid; L.ldr = ldr;
  L.gamma = gamma; L.M = M; L.N = N; L.K = K; L.stream = static_cast<cudaStream_t>(stream);
  rc = gemm_small_launch(L, P);
  if (rc == QVGGT_OK) count_launch(1);
  return rc;
}

int qvggt_w8a8_gemm(const int8_t* in, const int8_t* w, const void* wscales, const void* ascales, const void* bias,
                    void* out, int64_t M, int64_t N, int64_t K, void* stream) {
  GemmLaunch L;
  L.mode = B_I8;
  L.epi = EPI_STORE;
  L.a = in; L.lda = K; L.b = w; L.bias = bias; L.out = out; L.ldo = N; L.wscale = wscales; L.ascale = ascales;
  L.M = M; L.N = N; L.K = K; L.stream = static_cast<cudaStream_t>(stream);
  int rc = gemm_launch(L);
  if (rc == QVGGT_OK && M > 0) count_launch(1);
  return rc;
}

int qvggt_w8a8_gemm_residual(const int8_t* in, const int8_t* w, const void* wscales, const void* ascales,
                             const void* bias, const void* gamma, void* resid, int64_t M, int64_t N, int64_t K,
                             void* stream) {
  GemmLaunch L;
  L.mode = B_I8;
  L.epi = EPI_RESID;
  L.a = in; L.lda = K; L.b = w; L.bias = bias; L.out = resid; L.ldo = N; L.resid = resid; L.ldr = N;
  L.gamma = gamma; L.wscale = wscales; L.ascale = ascales;
  L.M = M; L.N = N; L.K = K; L.stream = static_cast<cudaStream_t>(stream);
  int rc = gemm_launch(L);
  if (rc == QVGGT_OK && M > 0) count_launch(1);
  return rc;
}

int qvggt_i8_gemm_i32(const int8_t* in, const int8_t* w, int32_t* acc, int64_t M, int64_t N, int64_t K,
                      void* stream) {
  GemmLaunch L;
  L.mode = B_I8;
  L.epi = EPI_I32;
  L.a = in; L.lda = K; L.b = w; L.out = acc; L.ldo = N;
  L.M = M; L.N = N; L.K = K; L.stream = static_cast<cudaStream_t>(stream);
  int rc = gemm_launch(L);
  if (rc == QVGGT_OK && M > 0) count_launch(1);
  return rc;
}

}  // extern "C"
