// fp32 SIMT fused GAT forward: every layer and both heads in one launch, with
// the node activations of a CTA's graphs resident in shared memory between
// layers.  This is the fp32 path (the TicTacToe configuration computes in
// fp32) and the generic path for every game.
//
// Per layer (networks/gat/gat.cu:836-870 names the stages; the math is the
// standard GAT the reference never completed):
//   Wh = X W_l                       one thread per output column, all rows
//   s_i^h = a_self^h . Wh_i^h,  t_j^h = a_nbr^h . Wh_j^h
//   e_ij = LeakyReLU_0.2(s_i + t_j) over CSR neighbours j of i
//   alpha = softmax_j(e_ij)
//   X_i = ELU(sum_j alpha_ij Wh_j + b_l)
// Heads (networks/gat/gat.cu:916-948 compute_output, 995-1031 softmax,
// 1033-1038 tanh): value = tanh(w2 . ReLU(W1^T mean_i X_i + b1) + b2); policy
// per game (TicTacToe per node 256->1, Connect4 column mean-pool 256->1, chess
// per node 256->73), then a softmax over all actions.
#include <cuda_runtime.h>
#include <stdint.h>

#include "gz_games.h"
#include "gz_internal.h"

namespace gz {
namespace {

constexpr int kThreads = 256;  // one thread per hidden column

template <int G> struct SimtCfg;
template <> struct SimtCfg<kConnect4> { static constexpr int GPC = 1; };  // graphs per CTA (TicTacToe: gat_simt_ttt.cu)
template <> struct SimtCfg<kChess> { static constexpr int GPC = 1; };

template <int G> struct SimtSmem {
  using T = Traits<G>;
  static constexpr int GPC = SimtCfg<G>::GPC;
  static constexpr int R = GPC * T::N;
  static constexpr size_t x = 0;                                        // X  [R][256]
  static constexpr size_t wh = x + (size_t)R * kHidden * 4;             // Wh [R][256]
  static constexpr size_t alpha = wh + (size_t)R * kHidden * 4;         // [GPC][NNZ][8]
  static constexpr size_t ss = alpha + (size_t)GPC * T::NNZ * kHeads * 4;  // [R][8]
  static constexpr size_t sn = ss + (size_t)R * kHeads * 4;             // [R][8]
  static constexpr size_t csr = sn + (size_t)R * kHeads * 4;            // row_ptr[N+1], col[NNZ]
  static constexpr size_t side = csr + (size_t)(T::N + 1 + T::NNZ) * 4; // [GPC] int
  static constexpr size_t bytes = side + 16;
};

// Offsets (floats) into the fp32 weight blob (gat_layout order) as
// compile-time arithmetic: a GatLayout indexed by the layer lives in local
// memory.
template <int G> struct SimtOff {
  using T = Traits<G>;
  static constexpr int kLayer0 = T::F * kHidden + kHidden + 2 * kHeads * kHeadDim;
  static constexpr int kLayerN = kHidden * kHidden + kHidden + 2 * kHeads * kHeadDim;
  __host__ __device__ static constexpr int W(int l) { return l == 0 ? 0 : kLayer0 + (l - 1) * kLayerN; }
  __host__ __device__ static constexpr int b(int l) { return W(l) + (l == 0 ? T::F : kHidden) * kHidden; }
  __host__ __device__ static constexpr int a(int l) { return b(l) + kHidden; }
  static constexpr int w_pi = kLayer0 + (T::L - 1) * kLayerN, b_pi = w_pi + kHidden * T::P;
  static constexpr int W_v1 = b_pi + T::P, b_v1 = W_v1 + kHidden * kValueHidden;
  static constexpr int w_v2 = b_v1 + kValueHidden, b_v2 = w_v2 + kValueHidden;
};

__device__ __forceinline__ float lrelu(float x) { return x > 0.f ? x : kLeakySlope * x; }
__device__ __forceinline__ float elu(float x) { return x > 0.f ? x : expm1f(x); }

template <int G>
__global__ void __launch_bounds__(kThreads) gat_simt_kernel(const float* __restrict__ w, const int* __restrict__ csr_g,
                                                            const int8_t* __restrict__ boards,
                                                            const int8_t* __restrict__ side_g, int n,
                                                            float* __restrict__ pi, float* __restrict__ v) {
  using T = Traits<G>;
  using S = SimtSmem<G>;
  constexpr int N = T::N, R = S::R, GPC = S::GPC, NNZ = T::NNZ;
  extern __shared__ __align__(16) unsigned char smem[];
  float* X = (float*)(smem + S::x);
  float* Wh = (float*)(smem + S::wh);
  float* alpha = (float*)(smem + S::alpha);
  float* ss = (float*)(smem + S::ss);
  float* sn = (float*)(smem + S::sn);
  int* rp = (int*)(smem + S::csr);
  int* col = rp + N + 1;
  int* side = (int*)(smem + S::side);
  const int tid = threadIdx.x;
  const int g0 = blockIdx.x * GPC;
  using L = SimtOff<G>;

  for (int i = tid; i < N + 1 + NNZ; i += kThreads) rp[i] = csr_g[i];
  if (tid < GPC) side[tid] = g0 + tid < n ? (int)side_g[g0 + tid] : 1;
  __syncthreads();

  // Encode node features into X[r][0..F).
  for (int r = tid; r < R; r += kThreads) {
    int g = r / N, i = r % N;
    float f[T::F];
    int gi = g0 + g < n ? g0 + g : n - 1;
    encode_node(G, boards + (size_t)gi * T::BOARD, side[g], i, f);
    for (int k = 0; k < T::F; ++k) X[r * kHidden + k] = f[k];
  }
  __syncthreads();

  int fin = T::F;
  for (int l = 0; l < T::L; ++l) {
    const float* W = w + L::W(l);
    const float* bias = w + L::b(l);
    const float* a = w + L::a(l);
    // Wh[:, c] = X W[:, c]
    {
      const int c = tid;
      float acc[R];
#pragma unroll
      for (int r = 0; r < R; ++r) acc[r] = 0.f;
      // W[k][c] for 16 K steps at a time, the next 16 loaded while these are
      // used (an L2 round trip per K step otherwise); X read as 16-byte
      // broadcasts (rows are 1 KB apart); the FMA order is k ascending
      int k = 0;
      if (fin % 16 == 0) {
        float wn[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) wn[j] = __ldg(W + (size_t)j * kHidden + c);
        for (; k < fin; k += 16) {
          float wc[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) wc[j] = wn[j];
          if (k + 16 < fin) {
#pragma unroll
            for (int j = 0; j < 16; ++j) wn[j] = __ldg(W + (size_t)(k + 16 + j) * kHidden + c);
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
#pragma unroll
            for (int r = 0; r < R; ++r) {
              const float4 x = *(const float4*)(X + r * kHidden + k + 4 * q);
              acc[r] = fmaf(x.x, wc[4 * q], acc[r]);
              acc[r] = fmaf(x.y, wc[4 * q + 1], acc[r]);
              acc[r] = fmaf(x.z, wc[4 * q + 2], acc[r]);
              acc[r] = fmaf(x.w, wc[4 * q + 3], acc[r]);
            }
          }
        }
      }
      for (; k + 4 <= fin; k += 4) {
        const float w0 = __ldg(W + (size_t)k * kHidden + c), w1 = __ldg(W + (size_t)(k + 1) * kHidden + c);
        const float w2 = __ldg(W + (size_t)(k + 2) * kHidden + c), w3 = __ldg(W + (size_t)(k + 3) * kHidden + c);
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const float4 x = *(const float4*)(X + r * kHidden + k);
          acc[r] = fmaf(x.x, w0, acc[r]);
          acc[r] = fmaf(x.y, w1, acc[r]);
          acc[r] = fmaf(x.z, w2, acc[r]);
          acc[r] = fmaf(x.w, w3, acc[r]);
        }
      }
      for (; k < fin; ++k) {
        const float wk = __ldg(W + (size_t)k * kHidden + c);
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] = fmaf(X[r * kHidden + k], wk, acc[r]);
      }
#pragma unroll
      for (int r = 0; r < R; ++r) Wh[r * kHidden + c] = acc[r];
    }
    __syncthreads();
    // attention scores per (row, head)
    for (int t = tid; t < R * kHeads; t += kThreads) {
      int r = t / kHeads, h = t % kHeads;
      const float* x = Wh + r * kHidden + h * kHeadDim;
      float s0 = 0.f, s1 = 0.f;
#pragma unroll 8
      for (int d = 0; d < kHeadDim; ++d) {
        s0 = fmaf(__ldg(a + (h * 2 + 0) * kHeadDim + d), x[d], s0);
        s1 = fmaf(__ldg(a + (h * 2 + 1) * kHeadDim + d), x[d], s1);
      }
      ss[t] = s0;
      sn[t] = s1;
    }
    __syncthreads();
    // neighbour softmax per (graph, node, head)
    for (int t = tid; t < R * kHeads; t += kThreads) {
      int r = t / kHeads, h = t % kHeads;
      int g = r / N, i = r % N;
      float si = ss[t];
      float m = -INFINITY;
      for (int e = rp[i]; e < rp[i + 1]; ++e) m = fmaxf(m, lrelu(si + sn[(g * N + col[e]) * kHeads + h]));
      float z = 0.f;
      for (int e = rp[i]; e < rp[i + 1]; ++e) {
        float p = expf(lrelu(si + sn[(g * N + col[e]) * kHeads + h]) - m);
        alpha[(g * NNZ + e) * kHeads + h] = p;
        z += p;
      }
      float inv = 1.f / z;
      for (int e = rp[i]; e < rp[i + 1]; ++e) alpha[(g * NNZ + e) * kHeads + h] *= inv;
    }
    __syncthreads();
    // aggregation + bias + ELU -> X
    {
      const int c = tid, h = c / kHeadDim;
      const float bc = __ldg(bias + c);
      for (int r = 0; r < R; ++r) {
        int g = r / N, i = r % N;
        float acc = 0.f;
        for (int e = rp[i]; e < rp[i + 1]; ++e)
          acc = fmaf(alpha[(g * NNZ + e) * kHeads + h], Wh[(g * N + col[e]) * kHidden + c], acc);
        X[r * kHidden + c] = elu(acc + bc);
      }
    }
    __syncthreads();
    fin = kHidden;
  }

  // ---- heads ----  (Wh is free now; reuse it as scratch)
  float* pooled = Wh;                  // [GPC][256]
  float* hid = Wh + GPC * kHidden;     // [GPC][64]
  float* logits = hid + GPC * kValueHidden;  // [GPC][A]
  {
    const int c = tid;
    for (int g = 0; g < GPC; ++g) {
      float s = 0.f;
      for (int i = 0; i < N; ++i) s += X[(g * N + i) * kHidden + c];
      pooled[g * kHidden + c] = s * (1.0f / N);
    }
  }
  __syncthreads();
  for (int t = tid; t < GPC * kValueHidden; t += kThreads) {
    int g = t / kValueHidden, u = t % kValueHidden;
    float acc = __ldg(w + L::b_v1 + u);
    for (int c = 0; c < kHidden; ++c) acc = fmaf(pooled[g * kHidden + c], __ldg(w + L::W_v1 + (size_t)c * kValueHidden + u), acc);
    hid[t] = fmaxf(acc, 0.f);
  }
  // policy logits
  if (G == kTicTacToe) {
    for (int t = tid; t < GPC * N; t += kThreads) {
      float acc = __ldg(w + L::b_pi);
      for (int c = 0; c < kHidden; ++c) acc = fmaf(X[t * kHidden + c], __ldg(w + L::w_pi + c), acc);
      logits[t] = acc;  // A == N
    }
  } else if (G == kConnect4) {
    for (int t = tid; t < GPC * 7; t += kThreads) {
      int g = t / 7, cc = t % 7;
      float acc = 0.f;
      for (int c = 0; c < kHidden; ++c) {
        float m = 0.f;
        for (int r = 0; r < 6; ++r) m += X[(g * N + r * 7 + cc) * kHidden + c];
        acc = fmaf(m * (1.0f / 6.0f), __ldg(w + L::w_pi + c), acc);
      }
      logits[t] = acc + __ldg(w + L::b_pi);
    }
  } else {
    for (int t = tid; t < GPC * T::A; t += kThreads) {
      int g = t / T::A, a = t % T::A, i = a / 73, k = a % 73;
      float acc = __ldg(w + L::b_pi + k);
      for (int c = 0; c < kHidden; ++c) acc = fmaf(X[(g * N + i) * kHidden + c], __ldg(w + L::w_pi + (size_t)c * 73 + k), acc);
      logits[t] = acc;
    }
  }
  __syncthreads();
  // softmax over actions and the value output: one warp per graph
  const int warp = tid / 32, lane = tid % 32;
  for (int g = warp; g < GPC; g += kThreads / 32) {
    int gi = g0 + g;
    float* lg = logits + g * T::A;
    float m = -INFINITY;
    for (int a = lane; a < T::A; a += 32) m = fmaxf(m, lg[a]);
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float z = 0.f;
    for (int a = lane; a < T::A; a += 32) z += expf(lg[a] - m);
    for (int o = 16; o; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
    float inv = 1.f / z;
    float vv = 0.f;
    for (int u = lane; u < kValueHidden; u += 32) vv = fmaf(hid[g * kValueHidden + u], __ldg(w + L::w_v2 + u), vv);
    for (int o = 16; o; o >>= 1) vv += __shfl_xor_sync(0xffffffffu, vv, o);
    if (gi < n) {
      for (int a = lane; a < T::A; a += 32) pi[(size_t)gi * T::A + a] = expf(lg[a] - m) * inv;
      if (lane == 0) v[gi] = tanhf(vv + __ldg(w + L::b_v2));
    }
  }
}

template <int G>
cudaError_t launch(const float* w, const int* csr, const int8_t* boards, const int8_t* side, int n, float* pi, float* v,
                   cudaStream_t stream) {
  using S = SimtSmem<G>;
  static_assert(S::bytes <= 227 * 1024, "shared memory budget");
  cudaError_t e = cudaFuncSetAttribute(gat_simt_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::bytes);
  if (e != cudaSuccess) return e;
  int grid = (n + S::GPC - 1) / S::GPC;
  gat_simt_kernel<G><<<grid, kThreads, S::bytes, stream>>>(w, csr, boards, side, n, pi, v);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gat_simt(int game, const float* w, const int* csr, const int8_t* boards, const int8_t* side, int n,
                            float* pi, float* v, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  switch (game) {
    case kTicTacToe: return launch_gat_simt_ttt(w, boards, side, n, pi, v, stream);
    case kConnect4: return launch<kConnect4>(w, csr, boards, side, n, pi, v, stream);
    case kChess: return launch<kChess>(w, csr, boards, side, n, pi, v, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace gz
