// C ABI entry points (include/b2msl.h): argument validation, path selection
// and error reporting. Validation is complete before any launch, so a failing
// call never leaves partial work on the stream.
#include <cstdarg>
#include <cstring>
#include <mutex>

#include "b2_common.cuh"

namespace b2 {

// kernels (defined in the family translation units)
int fa_simt_launch(const void*, const void*, const void*, void*, long long, long long, long long,
                   long long, const int64_t*, float, int, int, cudaStream_t);
bool fa_sm100_eligible(const void*, const void*, const void*, const void*, long long,
                       const int64_t*, int);
int fa_sm100_launch(const void*, const void*, const void*, void*, long long, long long, long long,
                    long long, const int64_t*, float, int, int, cudaStream_t);
int gemm_simt_launch(const void*, const void*, const void*, void*, long long, long long, long long,
                     const int64_t*, float, int, int, int, int, cudaStream_t);
bool gemm_sm100_eligible(const void*, const void*, long long, long long, long long,
                         const int64_t*, int);
int gemm_sm100_launch(const void*, const void*, const void*, void*, long long, long long,
                      long long, const int64_t*, float, int, int, int, int, void*, size_t, cudaStream_t,
                      int*);
size_t gemm_f16_workspace(long long, long long, long long, int);
size_t gemm_tf32x3_workspace(long long, long long, long long);
int gemm_tf32x3_launch(const float*, const float*, const void*, void*, long long, long long,
                       long long, const int64_t*, float, int, int, int, void*, cudaStream_t);
size_t row_op_workspace(int, long long, long long);
int row_op_launch(int, const void*, const void*, const void*, void*, long long, long long,
                  long long, long long, float, int, void*, size_t, cudaStream_t);
int gemm_stall_test_launch(const void*, const void*, void*, long long, long long, long long,
                           unsigned long long, cudaStream_t);
size_t axis_reduce_workspace(long long, long long, long long);
int axis_reduce_launch(int, const void*, void*, long long, long long, long long, int, void*, size_t,
                       cudaStream_t);
uint32_t row_read_status(bool);
uint32_t gemm_read_status(bool);
uint32_t pair_read_status(bool);
uint32_t fa_read_status(bool);

namespace {
thread_local std::string t_err;
thread_local const char* t_kernel = "";

// Tensor-core kernels need an sm_100-class device; remember per device.
constexpr int kMaxDev = 64;
int g_cc_major[kMaxDev];
std::once_flag g_cc_once[kMaxDev];

bool device_is_sm100() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return false;
  std::call_once(g_cc_once[dev], [dev] {
    int major = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    g_cc_major[dev] = major;
  });
  return g_cc_major[dev] == 10;
}

int g_sm_count[kMaxDev];
std::once_flag g_sm_once[kMaxDev];

bool valid_float_dtype(int dt) { return dt == B2_F32 || dt == B2_F16 || dt == B2_BF16; }
}  // namespace

void set_error(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_err = buf;
}
void clear_error() { t_err.clear(); }

namespace {
thread_local EpiProgram t_epi = {};
}
const EpiProgram& epi_program() { return t_epi; }
void set_epi_program(const EpiProgram* p) {
  if (p) t_epi = *p;
  else t_epi.n = 0;
}

int device_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return 148;
  std::call_once(g_sm_once[dev], [dev] {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_sm_count[dev] = n;
  });
  return g_sm_count[dev];
}

}  // namespace b2

using namespace b2;

extern "C" {

const char* b2_version(void) { return "b2msl 0.1.0 sm_100a"; }

const char* b2_last_error(void) { return t_err.c_str(); }

// Name of the kernel family the last successful call on this thread launched
// (test/bench introspection; not part of the reference surface).
const char* b2_last_kernel(void) { return t_kernel; }

int b2_fa_fwd(const void* q, const void* k, const void* v, void* o, int64_t B, int64_t H,
              int64_t S, int64_t D, const int64_t strides[16], float sm_scale, int causal,
              int dtype, void* stream) {
  clear_error();
  if (B < 0 || H < 0 || S < 0 || D <= 0) {
    set_error("b2_fa_fwd: invalid shape B=%lld H=%lld S=%lld D=%lld", (long long)B, (long long)H,
              (long long)S, (long long)D);
    return B2_EINVAL;
  }
  if (!valid_float_dtype(dtype)) {
    set_error("b2_fa_fwd: unsupported dtype %d", dtype);
    return B2_EINVAL;
  }
  if (B == 0 || H == 0 || S == 0) return B2_OK;
  if (!q || !k || !v || !o || !strides) {
    set_error("b2_fa_fwd: null pointer argument");
    return B2_EINVAL;
  }
  if (!(sm_scale == sm_scale) || sm_scale == INFINITY || sm_scale == -INFINITY) {
    set_error("b2_fa_fwd: sm_scale must be finite");
    return B2_EINVAL;
  }
  if (D > 128) {
    set_error("b2_fa_fwd: head_dim %lld > 128 is not supported", (long long)D);
    return B2_EUNSUPPORTED;
  }
  if (S >= (1LL << 31) || B * H >= (1LL << 31)) {
    set_error("b2_fa_fwd: S and B*H must be < 2^31");
    return B2_EINVAL;
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int rc;
  if (sm_scale > 0.f && device_is_sm100() && fa_sm100_eligible(q, k, v, o, D, strides, dtype)) {
    rc = fa_sm100_launch(q, k, v, o, B, H, S, D, strides, sm_scale, causal ? 1 : 0, dtype, st);
    if (rc == B2_OK) t_kernel = "fa_sm100";
  } else {
    rc = fa_simt_launch(q, k, v, o, B, H, S, D, strides, sm_scale, causal ? 1 : 0, dtype, st);
    if (rc == B2_OK) t_kernel = "fa_simt";
  }
  return rc;
}

namespace {
int gemm_impl(const void* A, const void* Bm, const void* bias, void* C, int64_t M, int64_t N,
              int64_t K, const int64_t strides[6], float alpha, int act, int in_dtype,
              int bias_dtype, int out_dtype, void* workspace, size_t ws_bytes, void* stream) {
  if (M < 0 || N < 0 || K < 0) {
    set_error("b2_gemm: invalid shape M=%lld N=%lld K=%lld", (long long)M, (long long)N, (long long)K);
    return B2_EINVAL;
  }
  if (!valid_float_dtype(in_dtype) || !valid_float_dtype(out_dtype) ||
      (bias && !valid_float_dtype(bias_dtype))) {
    set_error("b2_gemm: unsupported dtype combination in=%d bias=%d out=%d", in_dtype, bias_dtype,
              out_dtype);
    return B2_EINVAL;
  }
  if (act < B2_ACT_NONE || (act > B2_ACT_SOFTMAX && act != kActChain)) {
    set_error("b2_gemm: unknown activation %d", act);
    return B2_EINVAL;
  }
  if (M == 0 || N == 0) return B2_OK;
  if (!C || !strides || (K > 0 && (!A || !Bm))) {
    set_error("b2_gemm: null pointer argument");
    return B2_EINVAL;
  }
  if (act == B2_ACT_SOFTMAX && N > 256) {
    set_error("b2_gemm: the row-softmax epilogue needs N <= 256 (one output tile per row); got N=%lld",
              (long long)N);
    return B2_EUNSUPPORTED;
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int rc;
  const bool sm100 = device_is_sm100();
  // fp32 inputs: 3xTF32 on the tensor cores when the caller passed the
  // workspace b2_query_workspace asked for, else fp32 FMA.
  const size_t tf3_need = in_dtype == B2_F32 ? gemm_tf32x3_workspace(M, N, K) : 0;
  const bool tf3 = sm100 && in_dtype == B2_F32 && strides[5] == 1 && tf3_need > 0 && workspace &&
                   ws_bytes >= tf3_need && (reinterpret_cast<uintptr_t>(workspace) & 15) == 0;
  const bool tc = tf3 || (sm100 && strides[5] == 1 &&
                          gemm_sm100_eligible(A, Bm, M, N, K, strides, in_dtype));
  if (act == B2_ACT_SOFTMAX && !tc) {
    // CUDA-core path: fp32 logits into C, then the row-softmax kernel in place
    // (exact only when C holds fp32).
    if (out_dtype != B2_F32 || strides[5] != 1) {
      set_error("b2_gemm: row-softmax epilogue off the tensor-core path needs fp32, unit-stride C");
      return B2_EUNSUPPORTED;
    }
    rc = gemm_simt_launch(A, Bm, bias, C, M, N, K, strides, alpha, B2_ACT_NONE, in_dtype, bias_dtype,
                          out_dtype, st);
    if (rc != B2_OK) return rc;
    rc = row_op_launch(B2_ROW_SOFTMAX, C, nullptr, nullptr, C, M, N, strides[4], strides[4], 0.f,
                       B2_F32, nullptr, 0, st);
    if (rc == B2_OK) t_kernel = "gemm_simt+row_softmax";
    return rc;
  }
  if (tf3) {
    rc = gemm_tf32x3_launch(reinterpret_cast<const float*>(A), reinterpret_cast<const float*>(Bm),
                            bias, C, M, N, K, strides, alpha, act, bias_dtype, out_dtype, workspace, st);
    if (rc == B2_OK) t_kernel = "gemm_sm100_tf32x3";
  } else if (tc) {
    int variant = 0;
    rc = gemm_sm100_launch(A, Bm, bias, C, M, N, K, strides, alpha, act, in_dtype, bias_dtype,
                           out_dtype, workspace, ws_bytes, st, &variant);
    if (rc == B2_OK)
      t_kernel = variant == 3   ? "gemm_sm100_pair"
                 : variant == 2 ? "gemm_sm100_splitk"
                 : variant == 1 ? "gemm_sm100_n128"
                                : "gemm_sm100";
  } else {
    rc = gemm_simt_launch(A, Bm, bias, C, M, N, K, strides, alpha, act, in_dtype, bias_dtype,
                          out_dtype, st);
    if (rc == B2_OK) t_kernel = "gemm_simt";
  }
  return rc;
}

}  // namespace

int b2_gemm(const void* A, const void* Bm, const void* bias, void* C, int64_t M, int64_t N,
            int64_t K, const int64_t strides[6], float alpha, int act, int in_dtype,
            int bias_dtype, int out_dtype, void* workspace, size_t ws_bytes, void* stream) {
  clear_error();
  if (act == kActChain) {
    set_error("b2_gemm: unknown activation %d", act);
    return B2_EINVAL;
  }
  set_epi_program(nullptr);
  return gemm_impl(A, Bm, bias, C, M, N, K, strides, alpha, act, in_dtype, bias_dtype, out_dtype,
                   workspace, ws_bytes, stream);
}

int b2_gemm_epilogue(const void* A, const void* Bm, const void* bias, void* C, int64_t M, int64_t N,
                     int64_t K, const int64_t strides[6], const int32_t* codes, const float* args,
                     int n_ops, int in_dtype, int bias_dtype, int out_dtype, void* workspace,
                     size_t ws_bytes, void* stream) {
  clear_error();
  if (n_ops < 0 || n_ops > kMaxEpiOps || (n_ops > 0 && (!codes || !args))) {
    set_error("b2_gemm_epilogue: need 0 <= n_ops <= %d with codes and args", kMaxEpiOps);
    return B2_EINVAL;
  }
  EpiProgram prog = {};
  prog.n = n_ops;
  for (int i = 0; i < n_ops; ++i) {
    if (codes[i] < B2_EPI_ADD || codes[i] > B2_EPI_FMA) {
      set_error("b2_gemm_epilogue: unknown op code %d at position %d", codes[i], i);
      return B2_EINVAL;
    }
    if ((codes[i] == B2_EPI_ADD_BIAS || codes[i] == B2_EPI_MUL_BIAS) && !bias) {
      set_error("b2_gemm_epilogue: op %d at position %d needs a bias vector", codes[i], i);
      return B2_EINVAL;
    }
    prog.code[i] = codes[i];
    prog.a[i] = args[2 * i];
    prog.b[i] = args[2 * i + 1];
  }
  set_epi_program(&prog);
  const int rc = gemm_impl(A, Bm, bias, C, M, N, K, strides, 1.f, kActChain, in_dtype, bias_dtype,
                           out_dtype, workspace, ws_bytes, stream);
  set_epi_program(nullptr);
  return rc;
}

int b2_row_op(int op, const void* x, const void* w, const void* b, void* out, int64_t rows,
              int64_t cols, int64_t ld_x, int64_t ld_out, float eps, int dtype, void* workspace,
              size_t ws_bytes, void* stream) {
  clear_error();
  if (op < B2_ROW_SOFTMAX || op > B2_ROW_ARGMIN) {
    set_error("b2_row_op: unknown op %d", op);
    return B2_EINVAL;
  }
  if (!valid_float_dtype(dtype)) {
    set_error("b2_row_op: unsupported dtype %d", dtype);
    return B2_EINVAL;
  }
  if (rows < 0 || cols < 0) {
    set_error("b2_row_op: invalid shape rows=%lld cols=%lld", (long long)rows, (long long)cols);
    return B2_EINVAL;
  }
  const bool row_out = op == B2_ROW_SOFTMAX || op == B2_ROW_LAYERNORM || op == B2_ROW_RMSNORM;
  if (cols == 0 && (op == B2_ROW_MAX || op == B2_ROW_MIN || op == B2_ROW_ARGMAX || op == B2_ROW_ARGMIN) && rows > 0) {
    set_error("b2_row_op: max/min/argmax/argmin over an empty row is undefined");
    return B2_EINVAL;
  }
  if (rows == 0 || (cols == 0 && row_out)) return B2_OK;
  if (!out || (cols > 0 && !x)) {
    set_error("b2_row_op: null pointer argument");
    return B2_EINVAL;
  }
  if (ld_x < cols || (row_out && ld_out < cols)) {
    set_error("b2_row_op: row stride smaller than the row (ld_x=%lld ld_out=%lld cols=%lld)",
              (long long)ld_x, (long long)ld_out, (long long)cols);
    return B2_EINVAL;
  }
  if (rows >= (1LL << 31)) {
    set_error("b2_row_op: rows must be < 2^31");
    return B2_EINVAL;
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cols == 0) {  // sum over an empty row is 0
    const size_t bytes = (size_t)rows * dtype_size(dtype);
    B2_CUDA_TRY(cudaMemsetAsync(out, 0, bytes, st));
    t_kernel = "row_memset";
    return B2_OK;
  }
  const int rc = row_op_launch(op, x, w, b, out, rows, cols, ld_x, ld_out, eps, dtype, workspace,
                               ws_bytes, st);
  if (rc == B2_OK) t_kernel = row_op_workspace(op, rows, cols) ? "row_split" : "row_reduce";
  return rc;
}

int b2_reduce_axis(int op, const void* x, void* out, int64_t outer, int64_t R, int64_t inner,
                   int dtype, void* workspace, size_t ws_bytes, void* stream) {
  clear_error();
  if (op != B2_ROW_SUM && op != B2_ROW_MAX && op != B2_ROW_MIN && op != B2_ROW_ARGMAX &&
      op != B2_ROW_ARGMIN) {
    set_error("b2_reduce_axis: op %d is not sum/max/min/argmax/argmin", op);
    return B2_EINVAL;
  }
  if (!valid_float_dtype(dtype)) {
    set_error("b2_reduce_axis: unsupported dtype %d", dtype);
    return B2_EINVAL;
  }
  if (outer < 0 || R < 0 || inner < 0) {
    set_error("b2_reduce_axis: invalid shape outer=%lld R=%lld inner=%lld", (long long)outer,
              (long long)R, (long long)inner);
    return B2_EINVAL;
  }
  if (R == 0 && op != B2_ROW_SUM && outer * inner > 0) {
    set_error("b2_reduce_axis: max/min/argmax/argmin over an empty axis is undefined");
    return B2_EINVAL;
  }
  if (outer == 0 || inner == 0) return B2_OK;
  if (!out || (R > 0 && !x)) {
    set_error("b2_reduce_axis: null pointer argument");
    return B2_EINVAL;
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (R == 0) {  // sum over an empty axis is 0
    B2_CUDA_TRY(cudaMemsetAsync(out, 0, (size_t)(outer * inner) * dtype_size(dtype), st));
    t_kernel = "row_memset";
    return B2_OK;
  }
  const int rc = axis_reduce_launch(op, x, out, outer, R, inner, dtype, workspace, ws_bytes, st);
  if (rc == B2_OK) t_kernel = "axis_reduce";
  return rc;
}

size_t b2_query_workspace(int kind, int64_t a0, int64_t a1, int64_t a2, int64_t a3) {
  (void)a3;
  switch (kind) {
    case 0:
      if (!device_is_sm100()) return 0;
      if (a3 == B2_F32) return gemm_tf32x3_workspace(a0, a1, a2);
      return gemm_f16_workspace(a0, a1, a2, B2_ACT_NONE);
    case 1: return row_op_workspace((int)a0, a1, a2);
    case 2: return 0;
    case 3: return axis_reduce_workspace(a0, a1, a2);
    default: return 0;
  }
}

int b2_test_stalled_gemm(const void* A, const void* Bm, void* C, int64_t M, int64_t N, int64_t K,
                         uint64_t wait_limit_ns, void* stream) {
  clear_error();
  if (M <= 0 || N <= 0 || K <= 0 || M >= (1LL << 31) || N >= (1LL << 31) || K >= (1LL << 31) ||
      (K * 2) % 16 != 0) {
    set_error("b2_test_stalled_gemm: invalid shape M=%lld N=%lld K=%lld (K*2 must be a multiple of 16)",
              (long long)M, (long long)N, (long long)K);
    return B2_EINVAL;
  }
  if (!A || !Bm || !C || ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(Bm)) & 15)) {
    set_error("b2_test_stalled_gemm: null or unaligned operand");
    return B2_EINVAL;
  }
  if (wait_limit_ns == 0 || wait_limit_ns > kWaitLimitNs) {
    set_error("b2_test_stalled_gemm: wait limit must be in (0, %llu] ns", kWaitLimitNs);
    return B2_EINVAL;
  }
  if (!device_is_sm100()) {
    set_error("b2_test_stalled_gemm: needs an sm_100 device");
    return B2_EUNSUPPORTED;
  }
  const int rc = gemm_stall_test_launch(A, Bm, C, M, N, K, wait_limit_ns,
                                        reinterpret_cast<cudaStream_t>(stream));
  if (rc == B2_OK) t_kernel = "gemm_sm100";
  return rc;
}

int b2_device_status(int device, int clear, uint32_t* status_out) {
  clear_error();
  int prev = 0;
  B2_CUDA_TRY(cudaGetDevice(&prev));
  B2_CUDA_TRY(cudaSetDevice(device));
  cudaError_t e = cudaDeviceSynchronize();
  uint32_t s = 0;
  if (e == cudaSuccess) {
    s |= row_read_status(clear != 0);
    s |= gemm_read_status(clear != 0);
    s |= pair_read_status(clear != 0);
    s |= fa_read_status(clear != 0);
    e = cudaGetLastError();
  }
  cudaSetDevice(prev);
  if (e != cudaSuccess) {
    set_error("b2_device_status: %s", cudaGetErrorString(e));
    return B2_ELAUNCH;
  }
  if (status_out) *status_out = s;
  return s ? B2_ETIMEOUT : B2_OK;
}

}  // extern "C"
