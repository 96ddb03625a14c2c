// Equivariant linear maps: row addressing and launcher declarations.
#pragma once
#include "fc_base.cuh"

namespace fc {

template <typename T>
struct LinRows {
  const T* p;
  int64_t ld;   // elements between consecutive n
  int64_t off;  // offset of the rank block
  int64_t ms;   // elements between consecutive m
  int M;        // 2l+1
  FC_HD FC_INLINE const T* row(int64_t r) const {
    const int64_t n = r / M, m = r - n * M;
    return p + n * ld + off + m * ms;
  }
};

template <typename T>
struct LinGemmArgs {
  LinRows<T> a;     // A(r, k), k contiguous
  const T* w;       // weights of this rank
  int ldw;          // row length of W
  int trans_b;      // B(k, c) = trans_b ? W[c*ldw + k] : W[k*ldw + c]
  const T* scale;   // device pointer to the scale of this rank
  LinRows<T> c;     // C(r, col), col contiguous
  int64_t R;
  int K, N;
  // optional: the weights already split into tf32 hi | lo rows (n-major, k padded to a
  // multiple of 4), as lin_presplit writes them; null = split inside the call
  const T* bsplit = nullptr;
  // activation: 0 none; 1 C = (sW) silu(A) (forward); 2 C = silu'(aux) * (sW) A with aux
  // laid out like C (the backward's input gradient, aux = the forward's input); 3 C =
  // (sW) A + aux (a residual laid out like C, possibly C itself; TMA path only)
  int act = 0;
  LinRows<T> aux{};
};

template <typename T>
struct LinWgradArgs {
  LinRows<T> g;     // grad_out rows (col = out channel)
  LinRows<T> x;     // input rows (col = in channel)
  const T* scale;
  T* gw;            // (N_out, K_in) row-major
  int64_t R;
  int n_out, k_in;
  int64_t rows_per_split;
};

template <typename T>
int lin_gemm(const LinGemmArgs<T>& a, cudaStream_t s);
// fp32 on tcgen05 tensor cores: split = 3xTF32 (fp32 accuracy), else one tf32 product.
int lin_gemm_tc(const LinGemmArgs<float>& a, bool split, int* status, cudaStream_t s);
// TMA-fed persistent variant; returns 1 (nothing launched) when the layout is not eligible.
int lin_gemm_tma(const LinGemmArgs<float>& a, bool split, int* status, cudaStream_t s);
// all ranks of one map in one launch (uniform rank blocks, back to back); 1 = not eligible
int lin_gemm_tma_grouped(const LinGemmArgs<float>* a, int n, bool split, int* status, cudaStream_t s);
template <typename T>
int lin_wgrad(LinWgradArgs<T> a, cudaStream_t s);
// B(k, n) of a GEMM (W[n*ldw + k] if trans_b, else W[k*ldw + n]) as tf32 hi rows then lo
// rows, n-major with k padded to kp = (K + 3) & ~3 (zeros): 2 * N * kp floats at out.
int lin_presplit(const float* w, int ldw, int trans_b, int K, int N, float* out, cudaStream_t s);

}  // namespace fc
