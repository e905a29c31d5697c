// lq_sparse.cu -- sparse row correction of a linear layer's output.
//
// SpQRLinear.forward (spqr.py:172-197) dequantizes the int weight, writes the
// fp outlier values over the masked positions and calls F.linear.  With the
// int part done by the W4A16 kernel, the outliers are a sparse matrix C
// (C[n, k] = outlier - dequantized int weight at a masked (n, k)) whose
// product is added to y: y[m, n] += sum_k x[m, k] * C[n, k].  C is stored by
// rows (CSR over the rows that hold outliers); one thread owns one (m, row)
// pair, sums its row in fp32 and adds the sum to y with one rounding, so no
// two threads touch the same output.
#include "lq_common.cuh"

namespace lq {
namespace {

template <typename T>
__global__ void __launch_bounds__(256) sparse_row_add_kernel(const T* __restrict__ x, int64_t M,
                                                             int64_t K, int64_t N,
                                                             const int32_t* __restrict__ row_ptr,
                                                             const int32_t* __restrict__ row_ids,
                                                             int64_t n_rows,
                                                             const int32_t* __restrict__ cols,
                                                             const float* __restrict__ vals,
                                                             T* __restrict__ y) {
  const int64_t total = M * n_rows;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i % n_rows, m = i / n_rows;
    const T* xm = x + m * K;
    float acc = 0.0f;
    for (int32_t j = row_ptr[r]; j < row_ptr[r + 1]; ++j) acc = fmaf(Ty<T>::to_f(xm[cols[j]]), vals[j], acc);
    T* yp = y + m * N + row_ids[r];
    *yp = Ty<T>::from_f(__fadd_rn(Ty<T>::to_f(*yp), acc));
  }
}

template <typename T>
int sparse_row_add_t(const void* x, int64_t M, int64_t K, int64_t N, const int32_t* row_ptr,
                     const int32_t* row_ids, int64_t n_rows, const int32_t* cols, const float* vals,
                     void* y, cudaStream_t st) {
  const int64_t total = M * n_rows;
  int64_t want = (total + 255) / 256;
  const int64_t cap = (int64_t)num_sms() * 16;
  const int grid = (int)(want < 1 ? 1 : (want < cap ? want : cap));
  sparse_row_add_kernel<T><<<grid, 256, 0, st>>>(static_cast<const T*>(x), M, K, N, row_ptr, row_ids,
                                                  n_rows, cols, vals, static_cast<T*>(y));
  return launched("sparse_row_add_kernel");
}

}  // namespace
}  // namespace lq

using namespace lq;

extern "C" int lq_sparse_row_add(const void* x, int dtype, int64_t M, int64_t K, int64_t N,
                                 const int32_t* row_ptr, const int32_t* row_ids, int64_t n_rows,
                                 const int32_t* cols, const float* vals, void* y, void* stream) {
  LQ_REQUIRE(M >= 0 && K >= 0 && N >= 0 && n_rows >= 0, LQ_EINVAL, "bad size");
  if (M == 0 || n_rows == 0) return LQ_OK;
  LQ_REQUIRE(x && row_ptr && row_ids && cols && vals && y, LQ_EINVAL, "NULL pointer");
  cudaStream_t st = as_stream(stream);
  switch (dtype) {
    case LQ_F32: return sparse_row_add_t<float>(x, M, K, N, row_ptr, row_ids, n_rows, cols, vals, y, st);
    case LQ_F16: return sparse_row_add_t<__half>(x, M, K, N, row_ptr, row_ids, n_rows, cols, vals, y, st);
    case LQ_BF16: return sparse_row_add_t<__nv_bfloat16>(x, M, K, N, row_ptr, row_ids, n_rows, cols, vals, y, st);
    default: set_error("unsupported dtype %d", dtype); return LQ_EDTYPE;
  }
}
