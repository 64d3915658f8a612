// GAT training step: loss, backward pass, Adam, and the data-parallel
// gradient all-reduce.
//
// The reference trains through libtorch autograd and torch::optim::Adam
// (networks/gat/gat.cu:82-148 gat_train, 381-543 gat_train_distributed,
// 1040-1109 loss gradients: softmax cross-entropy gradient p - pi, value MSE
// gradient 2 (v - z)); its forward_gat is never defined (gat.cuh:103).  Here
// the step is written out by hand for the GAT the inference kernels compute:
//
//   loss = mean_b [ -sum_a pi_a log p_a + (z - v)^2 ]
//
// Forward (fp32, activations kept for the backward pass), per layer l:
//   Wh = X W_l                       GEMM over all B*N node rows
//   s_i = a_self . Wh_i^h, t_j = a_nbr . Wh_j^h, x_ij = s_i + t_j
//   alpha_ij = softmax_j lrelu(x_ij)  over the board graph's CSR neighbours
//   Y_i = sum_j alpha_ij Wh_j + b,  X' = ELU(Y)          (one CTA per position and group of heads)
// Backward, per layer (the same CTAs for the graph part):
//   dY = dX' * ELU'(Y); db = sum dY (per position, then over the batch)
//   dalpha_ij = dY_i . Wh_j; de_ij = alpha_ij (dalpha_ij - sum_k alpha_ik dalpha_ik)
//   dx_ij = de_ij lrelu'(x_ij); ds_i = sum_j dx_ij; dt_j = sum_i dx_ij
//   dWh_j = sum_i alpha_ij dY_i + ds_j a_self + dt_j a_nbr
//   da_self^h = sum_i ds_i Wh_i^h, da_nbr^h = sum_j dt_j Wh_j^h
//   dW_l = X^T dWh, dX = dWh W_l^T   (GEMMs, the first split over K)
// Every reduction runs in a fixed order (no floating-point atomics), so a
// step is bit-for-bit reproducible.  The graphs are symmetric, so the sums
// over a node's in-edges walk its CSR row through a reverse-edge table.
//
// Adam follows torch::optim::Adam with weight decay added to the gradient
// (gat.cu:71: lr 1e-3, weight decay 1e-4; betas 0.9 / 0.999, eps 1e-8).
// Gradients live in one flat buffer in the weight blob's layout, so the
// distributed step all-reduces contiguous buckets (one per layer, one for
// the heads) on a side stream as soon as the backward pass has produced
// them.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <vector>

#include "gz_games.h"
#include "gz_internal.h"
#include "gz_train.h"

namespace gz {
namespace train {

// ---------------------------------------------------------------- GEMM ----
// C[M x N] (+)= op(A)[M x K] . op(B)[K x N], row-major, fp32 on CUDA cores.
// op(A)(m, k) = ta ? A[k * lda + m] : A[m * lda + k]; likewise B.  A 64 x 64
// tile per CTA of 256 threads, 4 x 4 outputs per thread; blockIdx.z splits K
// (partial tiles go to `part`, summed in split order by gemm_reduce_kernel).
constexpr int kBM = 64, kBN = 64, kBK = 16;

__global__ void __launch_bounds__(256) gemm_kernel(int M, int N, int K, const float* __restrict__ A, int lda, int ta,
                                                   const float* __restrict__ B, int ldb, int tb, float* C, int ldc,
                                                   int accumulate, int k_chunk, float* part) {
  __shared__ float As[kBK][kBM + 4];
  __shared__ float Bs[kBK][kBN + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * kBN;
  const int k_lo = blockIdx.z * k_chunk, k_hi = min(K, k_lo + k_chunk);
  float acc[4][4] = {};
  for (int k0 = k_lo; k0 < k_hi; k0 += kBK) {
    for (int e = threadIdx.x; e < kBM * kBK; e += 256) {
      // element (m, k) of the A tile; consecutive threads walk the
      // contiguous dimension of A in memory
      int m, k;
      if (ta) { m = e % kBM; k = e / kBM; } else { k = e % kBK; m = e / kBK; }
      const int gm = m0 + m, gk = k0 + k;
      As[k][m] = (gm < M && gk < k_hi) ? (ta ? A[(size_t)gk * lda + gm] : A[(size_t)gm * lda + gk]) : 0.f;
    }
    for (int e = threadIdx.x; e < kBN * kBK; e += 256) {
      int n, k;
      if (tb) { k = e % kBK; n = e / kBK; } else { n = e % kBN; k = e / kBN; }
      const int gn = n0 + n, gk = k0 + k;
      Bs[k][n] = (gn < N && gk < k_hi) ? (tb ? B[(size_t)gn * ldb + gk] : B[(size_t)gk * ldb + gn]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kBK; ++k) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[k][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[k][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
  float* out = part ? part + (size_t)blockIdx.z * M * N : C;
  const int ld = part ? N : ldc;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gm = m0 + ty + 16 * i, gn = n0 + tx + 16 * j;
      if (gm < M && gn < N) {
        float* c = out + (size_t)gm * ld + gn;
        *c = (!part && accumulate) ? *c + acc[i][j] : acc[i][j];
      }
    }
}

// The same product for large outputs: a 128 x 128 tile per CTA of 256
// threads, 8 x 8 outputs per thread (rows 4 ty .. 4 ty + 3 and 64 + 4 ty ..,
// columns likewise with tx), K in steps of 8 through two shared-memory
// buffers (the next step's operands are loaded into registers while the
// current one is multiplied; one barrier per step).  Each output still sums
// its products in ascending k, one fused multiply-add at a time.
constexpr int kBM2 = 128, kBN2 = 128, kBK2 = 8, kPad2 = 4;

// Element (row, j) of the im2col matrix of a [rows][128] activation on the
// 6 x 7 board: j = tap * 128 + channel with taps (ky, kx) row-major, 0 where
// the tap leaves the board (the Connect4 ResNet's 3 x 3 convolutions).
__device__ __forceinline__ float im2col_at(const float* __restrict__ in, int row, int j) {
  const int tap = j >> 7, ci = j & 127;
  const int p = row % 42, r = p / 7 + tap / 3 - 1, c = p % 7 + tap % 3 - 1;
  return (r >= 0 && r < 6 && c >= 0 && c < 7) ? __ldg(in + (size_t)(row - p + r * 7 + c) * 128 + ci) : 0.f;
}

// kIm: 0 plain operands; 1 A is the im2col matrix of the activation A
// points at (ta false); 2 likewise for B (tb false).
template <int kIm>
__global__ void __launch_bounds__(256) gemm128_kernel(int M, int N, int K, const float* __restrict__ A, int lda,
                                                      int ta, const float* __restrict__ B, int ldb, int tb, float* C,
                                                      int ldc, int accumulate, int k_chunk, float* part) {
  __shared__ __align__(16) float As[2][kBK2][kBM2 + kPad2];
  __shared__ __align__(16) float Bs[2][kBK2][kBN2 + kPad2];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * kBM2, n0 = blockIdx.x * kBN2;
  const int k_lo = blockIdx.z * k_chunk, k_hi = min(K, k_lo + k_chunk);
  float ra[4], rb[4];
  // element r of this thread's share of the A (B) tile at K step k0: (m, k)
  // with consecutive threads along A's (B's) contiguous dimension
  auto load = [&](int k0) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int e = threadIdx.x + 256 * r;
      int m, k;
      if (ta) { m = e % kBM2; k = e / kBM2; } else { k = e % kBK2; m = e / kBK2; }
      const int gm = m0 + m, gk = k0 + k;
      if constexpr (kIm == 1)
        ra[r] = (gm < M && gk < k_hi) ? im2col_at(A, gm, gk) : 0.f;
      else
        ra[r] = (gm < M && gk < k_hi) ? (ta ? A[(size_t)gk * lda + gm] : A[(size_t)gm * lda + gk]) : 0.f;
      int n, kb;
      if (tb) { kb = e % kBK2; n = e / kBK2; } else { n = e % kBN2; kb = e / kBN2; }
      const int gn = n0 + n, gkb = k0 + kb;
      if constexpr (kIm == 2)
        rb[r] = (gn < N && gkb < k_hi) ? im2col_at(B, gkb, gn) : 0.f;
      else
        rb[r] = (gn < N && gkb < k_hi) ? (tb ? B[(size_t)gn * ldb + gkb] : B[(size_t)gkb * ldb + gn]) : 0.f;
    }
  };
  auto store = [&](int buf) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int e = threadIdx.x + 256 * r;
      if (ta) As[buf][e / kBM2][e % kBM2] = ra[r]; else As[buf][e % kBK2][e / kBK2] = ra[r];
      if (tb) Bs[buf][e % kBK2][e / kBK2] = rb[r]; else Bs[buf][e / kBN2][e % kBN2] = rb[r];
    }
  };
  float acc[8][8] = {};
  int buf = 0;
  if (k_lo < k_hi) {
    load(k_lo);
    store(0);
  }
  __syncthreads();
  for (int k0 = k_lo; k0 < k_hi; k0 += kBK2) {
    const bool more = k0 + kBK2 < k_hi;
    if (more) load(k0 + kBK2);
#pragma unroll
    for (int k = 0; k < kBK2; ++k) {
      const float4 a0 = *(const float4*)&As[buf][k][4 * ty], a1 = *(const float4*)&As[buf][k][64 + 4 * ty];
      const float4 b0 = *(const float4*)&Bs[buf][k][4 * tx], b1 = *(const float4*)&Bs[buf][k][64 + 4 * tx];
      const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    if (more) store(buf ^ 1);
    __syncthreads();
    buf ^= 1;
  }
  float* out = part ? part + (size_t)blockIdx.z * M * N : C;
  const int ld = part ? N : ldc;
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int gm = m0 + (i < 4 ? 4 * ty + i : 64 + 4 * ty + i - 4);
      const int gn = n0 + (j < 4 ? 4 * tx + j : 64 + 4 * tx + j - 4);
      if (gm < M && gn < N) {
        float* c = out + (size_t)gm * ld + gn;
        *c = (!part && accumulate) ? *c + acc[i][j] : acc[i][j];
      }
    }
}

__global__ void gemm_reduce_kernel(int M, int N, int splits, const float* __restrict__ part, float* C, int ldc,
                                   int accumulate) {
  const size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= (size_t)M * N) return;
  float s = 0.f;
  for (int z = 0; z < splits; ++z) s += part[(size_t)z * M * N + e];
  float* c = C + (e / N) * ldc + e % N;
  *c = accumulate ? *c + s : s;
}

// Streaming multiprocessors of the current device (queried once per device).
static int device_sms() {
  static int sms[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (sms[dev] == 0 && cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    cudaGetLastError();
    sms[dev] = 148;
  }
  return sms[dev];
}

bool gemm_big(int M, int N) { return M >= kBM2 && N >= kBN2; }

cudaError_t gemm(Workspace& ws, int M, int N, int K, const float* A, int lda, bool ta, const float* B, int ldb,
                 bool tb, float* C, int ldc, bool accumulate, cudaStream_t s, int im2col) {
  if (M <= 0 || N <= 0) return cudaSuccess;
  if (im2col && (!gemm_big(M, N) || (im2col == 1 && ta) || (im2col == 2 && tb))) return cudaErrorInvalidValue;
  // large outputs take the 128 x 128 tile kernel
  const bool big = M >= kBM2 && N >= kBN2;
  const int bm = big ? kBM2 : kBM, bn = big ? kBN2 : kBN, bk = big ? kBK2 : kBK;
  const int tiles = ((M + bm - 1) / bm) * ((N + bn - 1) / bn);
  // Split K when the output has fewer tiles than about two waves of CTAs
  // (four 64 x 64 or two 128 x 128 CTAs fit on an SM) and K is long (the weight gradients
  // dW = X^T dY, whose K is the batch's rows): at least 128 K per split.
  // The split depends on the shape only, and the partials are summed in
  // split order, so a step is reproducible.
  int splits = 1;
  const int target = (big ? 4 : 8) * device_sms();
  if (tiles < target && K >= 512) {
    splits = (target + tiles - 1) / tiles;
    const int max_splits = K / 128;
    splits = splits > max_splits ? max_splits : splits;
    if ((size_t)splits * M * N > ws.split_floats) splits = (int)(ws.split_floats / ((size_t)M * N));
    if (splits < 1) splits = 1;
  }
  int k_chunk = (K + splits - 1) / splits;
  k_chunk = (k_chunk + bk - 1) / bk * bk;
  splits = (K + k_chunk - 1) / k_chunk;
  if (splits < 1) splits = 1;
  dim3 grid((N + bn - 1) / bn, (M + bm - 1) / bm, splits);
  float* part = splits > 1 ? ws.split : nullptr;
  if (big && im2col == 1)
    gemm128_kernel<1><<<grid, 256, 0, s>>>(M, N, K, A, lda, ta, B, ldb, tb, C, ldc, accumulate, k_chunk, part);
  else if (big && im2col == 2)
    gemm128_kernel<2><<<grid, 256, 0, s>>>(M, N, K, A, lda, ta, B, ldb, tb, C, ldc, accumulate, k_chunk, part);
  else if (big)
    gemm128_kernel<0><<<grid, 256, 0, s>>>(M, N, K, A, lda, ta, B, ldb, tb, C, ldc, accumulate, k_chunk, part);
  else
    gemm_kernel<<<grid, 256, 0, s>>>(M, N, K, A, lda, ta, B, ldb, tb, C, ldc, accumulate, k_chunk,
                                     splits > 1 ? ws.split : nullptr);
  if (splits > 1) {
    const size_t total = (size_t)M * N;
    gemm_reduce_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(M, N, splits, ws.split, C, ldc, accumulate);
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------- column sums ----
// out[c] (+)= sum_r in[r * ld + c]: rows split into kColSlices slices, each
// summed in row order, then the slices in slice order.
constexpr int kColSlices = 64;

__global__ void colsum_partial_kernel(const float* __restrict__ in, int R, int C, int ld, float* __restrict__ part) {
  const int c = blockIdx.x * 32 + (threadIdx.x & 31);
  const int slice = blockIdx.y * 8 + (threadIdx.x >> 5);
  const int rows = (R + kColSlices - 1) / kColSlices;
  const int r0 = slice * rows, r1 = min(R, r0 + rows);
  if (c >= C) return;
  float s = 0.f;
  for (int r = r0; r < r1; ++r) s += in[(size_t)r * ld + c];
  part[(size_t)slice * C + c] = s;
}

__global__ void colsum_final_kernel(const float* __restrict__ part, int C, float* out, int accumulate, float scale) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  float s = 0.f;
  for (int z = 0; z < kColSlices; ++z) s += part[(size_t)z * C + c];
  out[c] = (accumulate ? out[c] : 0.f) + s * scale;
}

cudaError_t colsum(Workspace& ws, const float* in, int R, int C, int ld, float* out, bool accumulate,
                   cudaStream_t s, float scale) {
  if (C <= 0) return cudaSuccess;
  dim3 grid((C + 31) / 32, kColSlices / 8);
  colsum_partial_kernel<<<grid, 256, 0, s>>>(in, R, C, ld, ws.colsum);
  colsum_final_kernel<<<(C + 255) / 256, 256, 0, s>>>(ws.colsum, C, out, accumulate, scale);
  return cudaGetLastError();
}

// --------------------------------------------------------------- encode ----
__global__ void encode_kernel(int game, const int8_t* __restrict__ boards, const int8_t* __restrict__ side, int B,
                              float* __restrict__ X) {
  const GameShape sh = game_shape(game);
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= B * sh.nodes) return;
  const int b = r / sh.nodes, i = r % sh.nodes;
  float f[18];
  encode_node(game, boards + (size_t)b * sh.board_bytes, side[b], i, f);
  for (int k = 0; k < sh.features; ++k) X[(size_t)r * sh.features + k] = f[k];
}

// ------------------------------------------------------ graph attention ----
// One CTA per position and group of heads.  Per-node feature vectors sit in
// shared memory with an odd row stride, so threads that walk nodes hit
// distinct banks.

struct GraphArgs {
  const int* g;  // row_ptr[N + 1] | col[nnz] | rev[nnz]; rev[e] = index of the edge j -> i for e = i -> j
  int N, nnz;
};

__device__ __forceinline__ void load_graph(const GraphArgs& ga, int* rp, int* col, int* rev) {
  for (int k = threadIdx.x; k <= ga.N; k += blockDim.x) rp[k] = ga.g[k];
  for (int k = threadIdx.x; k < ga.nnz; k += blockDim.x) {
    col[k] = ga.g[ga.N + 1 + k];
    if (rev) rev[k] = ga.g[ga.N + 1 + ga.nnz + k];
  }
}

// The attention kernels take one position and HS of its 8 heads per CTA
// (32 threads a head): 8 at large batches, 2 when a batch has too few
// positions to fill the device.  Heads are independent here, and each
// head's sums run in the same order whatever HS is.
template <int HS>
__host__ __device__ constexpr int wh_stride() { return 32 * HS + 1; }  // odd: node walks hit distinct banks

template <int HS>
size_t attn_fwd_smem(int N, int nnz) {
  return (size_t)(N * wh_stride<HS>() + N * 16 + nnz * 8) * 4 + (size_t)(N + 1 + nnz) * 4;
}
template <int HS>
size_t attn_bwd_smem(int N, int nnz) {
  return (size_t)(2 * N * wh_stride<HS>() + N * 16 + nnz * 8 + N * 16) * 4 + (size_t)(N + 1 + 2 * nnz) * 4;
}

// Scores S [N][16] (s_i of heads 0-7, then t_i), attention weights alpha
// [nnz][8], pre-activation Y = sum_j alpha_ij Wh_j + b and X' = ELU(Y), for
// heads h0 .. h0 + HS - 1 (h0 = HS blockIdx.y) of position blockIdx.x.
template <int HS>
__global__ void __launch_bounds__(32 * HS) attn_fwd_kernel(GraphArgs ga, const float* __restrict__ Wh,
                                                           const float* __restrict__ a, const float* __restrict__ bias,
                                                           float* __restrict__ S, float* __restrict__ alpha,
                                                           float* __restrict__ Y, float* __restrict__ Xn) {
  constexpr int kF = 32 * HS, kW = wh_stride<HS>();
  extern __shared__ float sm[];
  const int N = ga.N, nnz = ga.nnz, b = blockIdx.x, h0 = HS * blockIdx.y;
  float* wh = sm;           // [N][kW]: this CTA's heads' features
  float* ss = wh + N * kW;  // [N][16]
  float* al = ss + N * 16;  // [nnz][8]
  int* rp = (int*)(al + nnz * 8);
  int* col = rp + N + 1;
  load_graph(ga, rp, col, nullptr);
  const float* whg = Wh + (size_t)b * N * 256 + 32 * h0;
  for (int e = threadIdx.x; e < N * kF; e += kF) wh[(e / kF) * kW + e % kF] = whg[(size_t)(e / kF) * 256 + e % kF];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, hw = h0 + warp;
  {
    const float as = a[hw * 64 + lane], an = a[hw * 64 + 32 + lane];  // a[h][0 self / 1 neighbour][d]
    for (int i = 0; i < N; ++i) {
      const float x = wh[i * kW + 32 * warp + lane];
      float p = x * as, q = x * an;
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) {
        p += __shfl_xor_sync(0xffffffffu, p, o);
        q += __shfl_xor_sync(0xffffffffu, q, o);
      }
      if (lane == 0) {
        ss[i * 16 + hw] = p;
        ss[i * 16 + 8 + hw] = q;
      }
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < N * 2 * HS; e += kF) {  // this CTA's score columns
    const int i = e / (2 * HS), c = e % (2 * HS), k = (c < HS ? 0 : 8) + h0 + c % HS;
    S[(size_t)b * N * 16 + i * 16 + k] = ss[i * 16 + k];
  }
  for (int t = threadIdx.x; t < N * HS; t += kF) {
    const int i = t % N, h = h0 + t / N;
    const float si = ss[i * 16 + h];
    float mx = -INFINITY;
    for (int e = rp[i]; e < rp[i + 1]; ++e) {
      const float x = si + ss[col[e] * 16 + 8 + h];
      mx = fmaxf(mx, x > 0.f ? x : kLeakySlope * x);
    }
    float z = 0.f;
    for (int e = rp[i]; e < rp[i + 1]; ++e) {
      const float x = si + ss[col[e] * 16 + 8 + h];
      const float ex = expf((x > 0.f ? x : kLeakySlope * x) - mx);
      al[e * 8 + h] = ex;
      z += ex;
    }
    for (int e = rp[i]; e < rp[i + 1]; ++e) {
      const float w = al[e * 8 + h] / z;
      al[e * 8 + h] = w;
      alpha[((size_t)b * nnz + e) * 8 + h] = w;
    }
  }
  __syncthreads();
  const int f = threadIdx.x, h = h0 + (f >> 5), gf = 32 * h0 + f;
  const float bf = bias[gf];
  for (int i = 0; i < N; ++i) {
    float acc = 0.f;
    for (int e = rp[i]; e < rp[i + 1]; ++e) acc = fmaf(al[e * 8 + h], wh[col[e] * kW + f], acc);
    const float y = acc + bf;
    const size_t o = ((size_t)b * N + i) * 256 + gf;
    Y[o] = y;
    Xn[o] = y > 0.f ? y : expm1f(y);
  }
}

// Backward of attn_fwd_kernel for one position and HS heads: from dX'
// (gradient of the layer output) to dWh, this position's share of the bias
// gradient db_part [256] (dY = dX' ELU'(Y) summed over its nodes in order)
// and of the attention-weight gradient, da_part [8][2][32].
template <int HS>
__global__ void __launch_bounds__(32 * HS) attn_bwd_kernel(GraphArgs ga, const float* __restrict__ dXn,
                                                           const float* __restrict__ Y, const float* __restrict__ Wh,
                                                           const float* __restrict__ S, const float* __restrict__ alpha,
                                                           const float* __restrict__ a, float* __restrict__ dWh,
                                                           float* __restrict__ db_part, float* __restrict__ da_part) {
  constexpr int kF = 32 * HS, kW = wh_stride<HS>();
  extern __shared__ float sm[];
  const int N = ga.N, nnz = ga.nnz, b = blockIdx.x, h0 = HS * blockIdx.y;
  float* dy = sm;             // [N][kW]
  float* wh = dy + N * kW;    // [N][kW]
  float* ss = wh + N * kW;    // [N][16]
  float* dx = ss + N * 16;    // [nnz][8]: dalpha, then d(s_i + t_j)
  float* dst = dx + nnz * 8;  // [N][16]: ds (heads 0-7), dt (8-15)
  int* rp = (int*)(dst + N * 16);
  int* col = rp + N + 1;
  int* rev = col + nnz;
  load_graph(ga, rp, col, rev);
  const size_t base = (size_t)b * N * 256 + 32 * h0;
  for (int e = threadIdx.x; e < N * kF; e += kF) {
    const size_t ge = base + (size_t)(e / kF) * 256 + e % kF;
    const float y = Y[ge];
    const float g = dXn[ge] * (y > 0.f ? 1.f : expf(y));
    dy[(e / kF) * kW + e % kF] = g;
    wh[(e / kF) * kW + e % kF] = Wh[ge];
  }
  for (int e = threadIdx.x; e < N * 16; e += kF) ss[e] = S[(size_t)b * N * 16 + e];
  __syncthreads();
  const float* alb = alpha + (size_t)b * nnz * 8;
  {
    float sb = 0.f;
    for (int i = 0; i < N; ++i) sb += dy[i * kW + threadIdx.x];
    db_part[(size_t)b * 256 + 32 * h0 + threadIdx.x] = sb;
  }
  // node i, head h: dalpha over i's edges, softmax and LeakyReLU backward
  for (int t = threadIdx.x; t < N * HS; t += kF) {
    const int i = t % N, hl = t / N, h = h0 + hl;
    const float* dyi = dy + i * kW + 32 * hl;
    float sbar = 0.f;
    for (int e = rp[i]; e < rp[i + 1]; ++e) {
      const float* whj = wh + col[e] * kW + 32 * hl;
      float d = 0.f;
#pragma unroll 8
      for (int k = 0; k < 32; ++k) d = fmaf(dyi[k], whj[k], d);
      dx[e * 8 + h] = d;
      sbar = fmaf(alb[e * 8 + h], d, sbar);
    }
    float ds = 0.f;
    const float si = ss[i * 16 + h];
    for (int e = rp[i]; e < rp[i + 1]; ++e) {
      const float de = alb[e * 8 + h] * (dx[e * 8 + h] - sbar);
      const float x = si + ss[col[e] * 16 + 8 + h];
      const float g = x > 0.f ? de : kLeakySlope * de;
      dx[e * 8 + h] = g;
      ds += g;
    }
    dst[i * 16 + h] = ds;
  }
  __syncthreads();
  // node j, head h: dt_j = sum over the edges i -> j
  for (int t = threadIdx.x; t < N * HS; t += kF) {
    const int j = t % N, h = h0 + t / N;
    float dt = 0.f;
    for (int e = rp[j]; e < rp[j + 1]; ++e) dt += dx[rev[e] * 8 + h];
    dst[j * 16 + 8 + h] = dt;
  }
  __syncthreads();
  const int f = threadIdx.x, h = h0 + (f >> 5), d = f & 31;
  const float as = a[h * 64 + d], an = a[h * 64 + 32 + d];
  float pa = 0.f, pn = 0.f;
  for (int j = 0; j < N; ++j) {
    float acc = 0.f;
    for (int e = rp[j]; e < rp[j + 1]; ++e) acc = fmaf(alb[rev[e] * 8 + h], dy[col[e] * kW + f], acc);
    const float ds = dst[j * 16 + h], dt = dst[j * 16 + 8 + h];
    dWh[base + (size_t)j * 256 + f] = acc + ds * as + dt * an;
    const float w = wh[j * kW + f];
    pa = fmaf(ds, w, pa);
    pn = fmaf(dt, w, pn);
  }
  da_part[(size_t)b * 512 + h * 64 + d] = pa;
  da_part[(size_t)b * 512 + h * 64 + 32 + d] = pn;
}

// ---------------------------------------------------------------- heads ----
// Node mean over the position (value head input) and, for Connect4, the
// mean over each board column's 6 nodes (policy head input).
__global__ void pool_fwd_kernel(int game, const float* __restrict__ X, float* __restrict__ gmean,
                                float* __restrict__ colmean) {
  const GameShape sh = game_shape(game);
  const int b = blockIdx.x, f = threadIdx.x, N = sh.nodes;
  const float* x = X + (size_t)b * N * 256 + f;
  float tot = 0.f;
  for (int i = 0; i < N; ++i) tot += x[(size_t)i * 256];
  gmean[(size_t)b * 256 + f] = tot / (float)N;
  if (game == kConnect4)
    for (int c = 0; c < 7; ++c) {
      float s = 0.f;
      for (int r = 0; r < 6; ++r) s += x[(size_t)(r * 7 + c) * 256];
      colmean[((size_t)b * 7 + c) * 256 + f] = s / 6.f;
    }
}

__device__ __forceinline__ float block_sum(float x, float* red) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = x;
  __syncthreads();
  float s = 0.f;
  for (int k = 0; k < (int)(blockDim.x >> 5); ++k) s += red[k];
  return s;
}

__device__ __forceinline__ float block_max(float x, float* red) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = x;
  __syncthreads();
  float m = -INFINITY;
  for (int k = 0; k < (int)(blockDim.x >> 5); ++k) m = fmaxf(m, red[k]);
  return m;
}

// Per position: softmax cross-entropy of the policy logits (GEMM output
// without the bias) against pi, squared error of the value against z, and
// the gradients of loss / B with respect to the logits (dlog) and the value
// head's hidden pre-activation (dz1) and output pre-activation (dvpre).
__global__ void __launch_bounds__(256) loss_kernel(int game, const float* __restrict__ w, GatLayout t,
                                                   const float* __restrict__ logits, const float* __restrict__ z1,
                                                   const float* __restrict__ pi, const float* __restrict__ vt,
                                                   float inv_batch, float* __restrict__ dlog, float* __restrict__ dz1,
                                                   float* __restrict__ dvpre, float* __restrict__ hid,
                                                   float* __restrict__ terms) {
  __shared__ float red[8];
  const GameShape sh = game_shape(game);
  const int b = blockIdx.x, A = sh.actions, P = sh.policy_out;
  const float* lg = logits + (size_t)b * A;
  const float* tp = pi + (size_t)b * A;
  float mx = -INFINITY;
  for (int k = threadIdx.x; k < A; k += blockDim.x) mx = fmaxf(mx, lg[k] + w[t.b_pi + k % P]);
  mx = block_max(mx, red);
  float se = 0.f, st = 0.f;
  for (int k = threadIdx.x; k < A; k += blockDim.x) {
    se += expf(lg[k] + w[t.b_pi + k % P] - mx);
    st += tp[k];
  }
  se = block_sum(se, red);
  st = block_sum(st, red);
  const float logz = mx + logf(se);
  float ce = 0.f;
  for (int k = threadIdx.x; k < A; k += blockDim.x) {
    const float a = lg[k] + w[t.b_pi + k % P];
    ce += tp[k] * (logz - a);
    dlog[(size_t)b * A + k] = (expf(a - logz) * st - tp[k]) * inv_batch;
  }
  ce = block_sum(ce, red);
  // value head: 64 hidden units on threads 0..63
  const int u = threadIdx.x;
  float zz = 0.f, r = 0.f;
  if (u < kValueHidden) {
    zz = z1[(size_t)b * kValueHidden + u] + w[t.b_v1 + u];
    r = fmaxf(zz, 0.f);
    hid[(size_t)b * kValueHidden + u] = r;
  }
  const float vpre = block_sum(u < kValueHidden ? r * w[t.w_v2 + u] : 0.f, red) + w[t.b_v2];
  const float v = tanhf(vpre), z = vt[b];
  const float g = 2.f * (v - z) * (1.f - v * v) * inv_batch;
  if (u < kValueHidden) dz1[(size_t)b * kValueHidden + u] = zz > 0.f ? g * w[t.w_v2 + u] : 0.f;
  if (threadIdx.x == 0) {
    dvpre[b] = g;
    terms[(size_t)b * 2] = ce;
    terms[(size_t)b * 2 + 1] = (z - v) * (z - v);
  }
}

// dX of the last layer: the value head's mean-pool plus the policy input
// (Connect4: column means; TicTacToe and chess: the nodes themselves).
__global__ void pool_bwd_kernel(int game, const float* __restrict__ dgmean, const float* __restrict__ dpol,
                                float* __restrict__ dX) {
  const GameShape sh = game_shape(game);
  const int b = blockIdx.x, f = threadIdx.x, N = sh.nodes;
  const float g = dgmean[(size_t)b * 256 + f] / (float)N;
  for (int i = 0; i < N; ++i) {
    const float p = game == kConnect4 ? dpol[((size_t)b * 7 + i % 7) * 256 + f] / 6.f : dpol[((size_t)b * N + i) * 256 + f];
    dX[((size_t)b * N + i) * 256 + f] = g + p;
  }
}

// ----------------------------------------------------------------- Adam ----
// torch::optim::Adam (L2 weight decay added to the gradient):
//   g = grad * grad_scale + wd * w;  m = b1 m + (1 - b1) g;  v = b2 v + (1 - b2) g^2
//   w -= lr / (1 - b1^t) * m / (sqrt(v) / sqrt(1 - b2^t) + eps)
__global__ void adam_kernel(size_t n, float* __restrict__ w, const float* __restrict__ grad, float* __restrict__ m,
                            float* __restrict__ v, AdamParams p, float bc1, float bc2_sqrt) {
  const size_t k = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= n) return;
  const float g = grad[k] * p.grad_scale + p.weight_decay * w[k];
  const float mk = p.beta1 * m[k] + (1.f - p.beta1) * g;
  const float vk = p.beta2 * v[k] + (1.f - p.beta2) * g * g;
  m[k] = mk;
  v[k] = vk;
  w[k] -= (p.lr / bc1) * mk / (sqrtf(vk) / bc2_sqrt + p.eps);
}

// --------------------------------------------------------------- driver ----
// Buffers of a batch of up to B positions, offsets in floats into the arena.
struct Layout {
  size_t X[9];                            // X[0]: features [B*N][F]; X[l]: layer l's input [B*N][256]
  size_t Wh[8], Y[8], S[8], alpha[8];     // per layer
  size_t gmean, colmean, z1, logits, dlog, dz1, dvpre, hid, terms, dgmean, dpol, dXa, dXb, dWh, dbpart, dapart;
  size_t total;
};

Layout layout(int game, int B) {
  const GameShape sh = game_shape(game);
  const size_t N = sh.nodes, rows = (size_t)B * N, node_vec = rows * 256;
  const size_t pol_rows = game == kConnect4 ? (size_t)B * 7 : rows;
  Layout o{};
  size_t p = 0;
  auto take = [&](size_t n) {
    const size_t at = p;
    p += (n + 63) & ~(size_t)63;  // 256-byte aligned parts
    return at;
  };
  o.X[0] = take(rows * sh.features);
  for (int l = 1; l <= sh.layers; ++l) o.X[l] = take(node_vec);
  for (int l = 0; l < sh.layers; ++l) {
    o.Wh[l] = take(node_vec);
    o.Y[l] = take(node_vec);
    o.S[l] = take(rows * 16);
    o.alpha[l] = take((size_t)B * sh.nnz * 8);
  }
  o.gmean = take((size_t)B * 256);
  o.colmean = take((size_t)B * 7 * 256);
  o.z1 = take((size_t)B * kValueHidden);
  o.logits = take((size_t)B * sh.actions);
  o.dlog = take((size_t)B * sh.actions);
  o.dz1 = take((size_t)B * kValueHidden);
  o.dvpre = take(B);
  o.hid = take((size_t)B * kValueHidden);
  o.terms = take((size_t)B * 2);
  o.dgmean = take((size_t)B * 256);
  o.dpol = take(pol_rows * 256);
  o.dXa = take(node_vec);
  o.dXb = take(node_vec);
  o.dWh = take(node_vec);
  o.dbpart = take((size_t)B * 256);
  o.dapart = take((size_t)B * 512);
  o.total = p;
  return o;
}

int bucket_count(int game) { return game_shape(game).layers + 1; }

void bucket_range(int game, int k, size_t* offset, size_t* count) {
  const GatLayout t = gat_layout(game);
  if (k < t.L) {
    *offset = t.W[k];
    *count = t.a[k] + kHeads * 2 * kHeadDim - t.W[k];
  } else {
    *offset = t.w_pi;
    *count = t.total - t.w_pi;
  }
}

void free_state(State& st) {
  cudaFree(st.m);
  cudaFree(st.v);
  cudaFree(st.grad);
  cudaFree(st.loss);
  cudaFree(st.graph);
  cudaFree(st.ws.split);
  cudaFree(st.ws.colsum);
  cudaFree(st.arena);
  if (st.comm_stream) cudaStreamDestroy(st.comm_stream);
  for (auto& e : st.ev_bucket)
    if (e) cudaEventDestroy(e);
  if (st.ev_comm) cudaEventDestroy(st.ev_comm);
  st = State{};
}

cudaError_t ensure_state(State& st, int game, int capacity) {
  cudaError_t e = cudaSuccess;
  const GameShape sh = game_shape(game);
  if (st.game != game || st.kind != 0) {
    free_state(st);
    st.game = game;
    st.weight_count = gat_layout(game).total;
    const size_t wc = st.weight_count;
    if ((e = cudaMalloc(&st.m, wc * 4)) || (e = cudaMalloc(&st.v, wc * 4)) || (e = cudaMalloc(&st.grad, wc * 4)) ||
        (e = cudaMalloc(&st.loss, 2 * 4)))
      return e;
    if ((e = cudaMemset(st.m, 0, wc * 4)) || (e = cudaMemset(st.v, 0, wc * 4)) || (e = cudaMemset(st.grad, 0, wc * 4)))
      return e;
    // board graph with its reverse-edge table (the graphs are symmetric)
    std::vector<int> g(sh.nodes + 1 + 2 * sh.nnz);
    int* rp = g.data();
    int* col = rp + sh.nodes + 1;
    int* rev = col + sh.nnz;
    build_graph_csr(game, rp, col);
    for (int i = 0; i < sh.nodes; ++i)
      for (int e2 = rp[i]; e2 < rp[i + 1]; ++e2) {
        const int j = col[e2];
        rev[e2] = -1;
        for (int k = rp[j]; k < rp[j + 1]; ++k)
          if (col[k] == i) rev[e2] = k;
        if (rev[e2] < 0) return cudaErrorInvalidValue;  // not symmetric
      }
    if ((e = cudaMalloc(&st.graph, g.size() * 4)) ||
        (e = cudaMemcpy(st.graph, g.data(), g.size() * 4, cudaMemcpyHostToDevice)))
      return e;
    st.ws.split_floats = (size_t)4 << 20;
    if ((e = cudaMalloc(&st.ws.split, st.ws.split_floats * 4)) || (e = cudaMalloc(&st.ws.colsum, kColsumFloats * 4)))
      return e;
    if ((e = cudaStreamCreateWithFlags(&st.comm_stream, cudaStreamNonBlocking))) return e;
    for (auto& ev : st.ev_bucket)
      if ((e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming))) return e;
    if ((e = cudaEventCreateWithFlags(&st.ev_comm, cudaEventDisableTiming))) return e;
    // the kernels serve every game: allow the largest (chess) shared memory
    const GameShape big = game_shape(kChess);
    if ((e = cudaFuncSetAttribute(attn_fwd_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)attn_fwd_smem<8>(big.nodes, big.nnz))) ||
        (e = cudaFuncSetAttribute(attn_bwd_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)attn_bwd_smem<8>(big.nodes, big.nnz))) ||
        (e = cudaFuncSetAttribute(attn_fwd_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)attn_fwd_smem<2>(big.nodes, big.nnz))) ||
        (e = cudaFuncSetAttribute(attn_bwd_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)attn_bwd_smem<2>(big.nodes, big.nnz))))
      return e;
  }
  if (capacity > st.capacity) {
    cudaFree(st.arena);
    st.arena = nullptr;
    st.capacity = 0;
    const Layout o = layout(game, capacity);
    if ((e = cudaMalloc(&st.arena, o.total * 4))) return e;
    st.arena_floats = o.total;
    st.capacity = capacity;
  }
  return cudaSuccess;
}

#define GZ_TRY(expr)                        \
  do {                                      \
    const cudaError_t e_ = (expr);          \
    if (e_ != cudaSuccess) return e_;       \
  } while (0)

cudaError_t loss_and_grad(State& st, const float* w, const int8_t* boards, const int8_t* side, const float* pi,
                          const float* v, int B, cudaStream_t s, const std::function<cudaError_t(int)>& bucket_done) {
  if (B <= 0 || B > st.capacity) return cudaErrorInvalidValue;
  const int game = st.game;
  const GameShape sh = game_shape(game);
  const GatLayout t = gat_layout(game);
  const int N = sh.nodes, L = sh.layers, P = t.P, rowsN = B * N;
  const Layout o = layout(game, st.capacity);
  float* ar = st.arena;
  float* g = st.grad;
  Workspace& ws = st.ws;
  const GraphArgs ga{st.graph, N, sh.nnz};
  // all 8 heads of a position per CTA, or 2 when the batch has fewer
  // positions than the device has SMs
  const bool split_heads = B < device_sms();
  auto attn_fwd = [&](int l) {
    if (split_heads)
      attn_fwd_kernel<2><<<dim3(B, 4), 64, attn_fwd_smem<2>(N, sh.nnz), s>>>(
          ga, ar + o.Wh[l], w + t.a[l], w + t.b[l], ar + o.S[l], ar + o.alpha[l], ar + o.Y[l], ar + o.X[l + 1]);
    else
      attn_fwd_kernel<8><<<dim3(B, 1), 256, attn_fwd_smem<8>(N, sh.nnz), s>>>(
          ga, ar + o.Wh[l], w + t.a[l], w + t.b[l], ar + o.S[l], ar + o.alpha[l], ar + o.Y[l], ar + o.X[l + 1]);
  };
  auto attn_bwd = [&](int l, const float* dX) {
    if (split_heads)
      attn_bwd_kernel<2><<<dim3(B, 4), 64, attn_bwd_smem<2>(N, sh.nnz), s>>>(
          ga, dX, ar + o.Y[l], ar + o.Wh[l], ar + o.S[l], ar + o.alpha[l], w + t.a[l], ar + o.dWh, ar + o.dbpart,
          ar + o.dapart);
    else
      attn_bwd_kernel<8><<<dim3(B, 1), 256, attn_bwd_smem<8>(N, sh.nnz), s>>>(
          ga, dX, ar + o.Y[l], ar + o.Wh[l], ar + o.S[l], ar + o.alpha[l], w + t.a[l], ar + o.dWh, ar + o.dbpart,
          ar + o.dapart);
  };

  // ---- forward ----
  encode_kernel<<<(rowsN + 255) / 256, 256, 0, s>>>(game, boards, side, B, ar + o.X[0]);
  for (int l = 0; l < L; ++l) {
    const int Fl = l ? kHidden : sh.features;
    GZ_TRY(gemm(ws, rowsN, kHidden, Fl, ar + o.X[l], Fl, false, w + t.W[l], kHidden, false, ar + o.Wh[l], kHidden,
                false, s));
    attn_fwd(l);
  }
  float* XL = ar + o.X[L];
  pool_fwd_kernel<<<B, 256, 0, s>>>(game, XL, ar + o.gmean, ar + o.colmean);
  const float* polin = game == kConnect4 ? ar + o.colmean : XL;
  const int prow = game == kConnect4 ? B * 7 : rowsN;
  GZ_TRY(gemm(ws, B, kValueHidden, kHidden, ar + o.gmean, kHidden, false, w + t.W_v1, kValueHidden, false, ar + o.z1,
              kValueHidden, false, s));
  GZ_TRY(gemm(ws, prow, P, kHidden, polin, kHidden, false, w + t.w_pi, P, false, ar + o.logits, P, false, s));
  loss_kernel<<<B, 256, 0, s>>>(game, w, t, ar + o.logits, ar + o.z1, pi, v, 1.f / (float)B, ar + o.dlog, ar + o.dz1,
                                ar + o.dvpre, ar + o.hid, ar + o.terms);
  GZ_TRY(colsum(ws, ar + o.terms, B, 2, 2, st.loss, false, s, 1.f / (float)B));

  // ---- heads backward ----
  GZ_TRY(gemm(ws, kValueHidden, 1, B, ar + o.hid, kValueHidden, true, ar + o.dvpre, 1, false, g + t.w_v2, 1, false, s));
  GZ_TRY(colsum(ws, ar + o.dvpre, B, 1, 1, g + t.b_v2, false, s));
  GZ_TRY(gemm(ws, kHidden, kValueHidden, B, ar + o.gmean, kHidden, true, ar + o.dz1, kValueHidden, false, g + t.W_v1,
              kValueHidden, false, s));
  GZ_TRY(colsum(ws, ar + o.dz1, B, kValueHidden, kValueHidden, g + t.b_v1, false, s));
  GZ_TRY(gemm(ws, kHidden, P, prow, polin, kHidden, true, ar + o.dlog, P, false, g + t.w_pi, P, false, s));
  GZ_TRY(colsum(ws, ar + o.dlog, prow, P, P, g + t.b_pi, false, s));
  GZ_TRY(gemm(ws, B, kHidden, kValueHidden, ar + o.dz1, kValueHidden, false, w + t.W_v1, kValueHidden, true,
              ar + o.dgmean, kHidden, false, s));
  GZ_TRY(gemm(ws, prow, kHidden, P, ar + o.dlog, P, false, w + t.w_pi, P, true, ar + o.dpol, kHidden, false, s));
  GZ_TRY(cudaGetLastError());
  GZ_TRY(bucket_done(L));

  // ---- layers backward ----
  float* dX = ar + o.dXa;
  float* dXn = ar + o.dXb;
  pool_bwd_kernel<<<B, 256, 0, s>>>(game, ar + o.dgmean, ar + o.dpol, dX);
  for (int l = L - 1; l >= 0; --l) {
    const int Fl = l ? kHidden : sh.features;
    attn_bwd(l, dX);
    GZ_TRY(colsum(ws, ar + o.dbpart, B, kHidden, kHidden, g + t.b[l], false, s));
    GZ_TRY(colsum(ws, ar + o.dapart, B, 512, 512, g + t.a[l], false, s));
    GZ_TRY(gemm(ws, Fl, kHidden, rowsN, ar + o.X[l], Fl, true, ar + o.dWh, kHidden, false, g + t.W[l], kHidden, false,
                s));
    if (l > 0) {
      GZ_TRY(gemm(ws, rowsN, kHidden, kHidden, ar + o.dWh, kHidden, false, w + t.W[l], kHidden, true, dXn, kHidden,
                  false, s));
      float* tmp = dX;
      dX = dXn;
      dXn = tmp;
    }
    GZ_TRY(cudaGetLastError());
    GZ_TRY(bucket_done(l));
  }
  return cudaSuccess;
}

cudaError_t adam_step(State& st, float* w, const AdamParams& p, cudaStream_t s) {
  st.step += 1;
  const double bc1 = 1.0 - pow((double)p.beta1, (double)st.step);
  const double bc2 = 1.0 - pow((double)p.beta2, (double)st.step);
  const size_t n = st.weight_count;
  adam_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(n, w, st.grad, st.m, st.v, p, (float)bc1,
                                                          (float)sqrt(bc2));
  return cudaGetLastError();
}

}  // namespace train
}  // namespace gz
