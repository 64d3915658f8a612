// fp32 SIMT GAT forward specialised for TicTacToe: the same math as
// gat_simt.cu (networks/gat/gat.cu:836-870 names the stages, 916-948 the
// heads), laid out for a 9-node graph.
//
// One CTA of 128 threads per position; thread t owns hidden columns
// 4j .. 4j + 3 (j = t % 64, head j / 8) of rows 0-4 (t < 64) or 5-8, so that
//   * the projection Wh = X W reads W as 16-byte rows (four columns per
//     load, sixteen K steps in flight) and each 16-byte broadcast of X feeds
//     four columns: 36 independent accumulators per thread;
//   * a head's attention scores are a sum over eight threads (shuffles);
//   * the graph is the 3x3 stencil (every node attends to itself and its
//     8-neighbourhood on the board), so the aggregation's neighbours are
//     compile-time constants: no index loads, all rows independent.
// Summation orders follow gat_simt.cu (k ascending, neighbours ascending).
#include <cuda_runtime.h>
#include <stdint.h>

#include "gz_games.h"
#include "gz_internal.h"

namespace gz {
namespace {

using TT = Traits<kTicTacToe>;
constexpr int kN = TT::N;   // 9 nodes
constexpr int kTT = 128;    // threads per position: 64 column groups x 2 row halves
constexpr int kHalf0 = 5;   // rows of the first half
constexpr int kSlots = 9;   // stencil slot (dr + 1) * 3 + (dc + 1)
static_assert(kHidden == 2 * kTT && kHeadDim == 32 && kHeads == 8, "thread j owns columns 4j..4j+3 of head j/8");

// Neighbour of node r in stencil slot s, or -1 off the board.
__host__ __device__ constexpr int stencil(int r, int s) {
  const int rr = r / 3 + s / 3 - 1, cc = r % 3 + s % 3 - 1;
  return rr >= 0 && rr < 3 && cc >= 0 && cc < 3 ? rr * 3 + cc : -1;
}

__device__ __forceinline__ float lrelu(float x) { return x > 0.f ? x : kLeakySlope * x; }
__device__ __forceinline__ float elu(float x) { return x > 0.f ? x : expm1f(x); }

// Offsets (floats) into the fp32 weight blob (gat_layout order), as
// compile-time arithmetic: a GatLayout indexed by the layer would live in
// local memory.
struct TttOff {
  static constexpr int kLayer0 = TT::F * kHidden + kHidden + 2 * kHeads * kHeadDim;
  static constexpr int kLayerN = kHidden * kHidden + kHidden + 2 * kHeads * kHeadDim;
  __host__ __device__ static constexpr int W(int l) { return l == 0 ? 0 : kLayer0 + (l - 1) * kLayerN; }
  __host__ __device__ static constexpr int b(int l) { return W(l) + (l == 0 ? TT::F : kHidden) * kHidden; }
  __host__ __device__ static constexpr int a(int l) { return b(l) + kHidden; }
  static constexpr int w_pi = kLayer0 + (TT::L - 1) * kLayerN, b_pi = w_pi + kHidden * TT::P;
  static constexpr int W_v1 = b_pi + TT::P, b_v1 = W_v1 + kHidden * kValueHidden;
  static constexpr int w_v2 = b_v1 + kValueHidden, b_v2 = w_v2 + kValueHidden;
};

struct TttSmem {
  float X[kN][kHidden];            // layer input / output
  float Wh[kN][kHidden];           // projection
  float ss[kN][kHeads], sn[kN][kHeads];
  float alpha[kN][kSlots][kHeads];  // softmax weights by stencil slot
  float pooled[kHidden];
  float hid[kValueHidden];
  float logit[kN];
  float red[2][kN + 1];             // per-warp partial sums of the policy logits (warps 0, 1)
};


// acc[i][c] += sum_k X[R0 + i][k] W[k][4j + c] over k < K, k ascending.  For
// K > 4 (a multiple of 16) W rows are loaded sixteen K steps ahead.
template <int R0, int NR, int K>
__device__ __forceinline__ void project(const float* __restrict__ W, const TttSmem& sm, int j, float (&acc)[kHalf0][4]) {
  const float4* Wj = (const float4*)W + j;  // row k: Wj[k * 64]
  auto step4 = [&](int k, const float4 (&w)[4]) {
#pragma unroll
    for (int i = 0; i < NR; ++i) {
      const float4 x = *(const float4*)&sm.X[R0 + i][k];
      const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc[i][0] = fmaf(xs[q], w[q].x, acc[i][0]);
        acc[i][1] = fmaf(xs[q], w[q].y, acc[i][1]);
        acc[i][2] = fmaf(xs[q], w[q].z, acc[i][2]);
        acc[i][3] = fmaf(xs[q], w[q].w, acc[i][3]);
      }
    }
  };
  if constexpr (K == 4) {
    float4 w[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) w[q] = __ldg(Wj + (size_t)q * 64);
    step4(0, w);
  } else {
    static_assert(K % 16 == 0, "K steps in groups of 16");
    float4 ring[4][4];  // slot s: rows k0 + 4 s .. k0 + 4 s + 3
#pragma unroll
    for (int s = 0; s < 4; ++s)
#pragma unroll
      for (int q = 0; q < 4; ++q) ring[s][q] = __ldg(Wj + (size_t)(4 * s + q) * 64);
    for (int k0 = 0; k0 < K; k0 += 16) {
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const int k = k0 + 4 * s;
        float4 w[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) w[q] = ring[s][q];
        if (k + 16 < K) {
#pragma unroll
          for (int q = 0; q < 4; ++q) ring[s][q] = __ldg(Wj + (size_t)(k + 16 + q) * 64);
        }
        step4(k, w);
      }
    }
  }
}

// Wh rows R0.. to shared memory and their attention scores: s_r^h =
// a_self^h . Wh_r^h and t_r^h = a_nbr^h . Wh_r^h summed over the head's
// eight threads (lanes 8 (h % 4) .. 8 (h % 4) + 7 of the warp).
template <int R0, int NR>
__device__ __forceinline__ void scores(const float* __restrict__ a, TttSmem& sm, int j, const float (&acc)[kHalf0][4]) {
  const int h = j >> 3;
  const float4 as = __ldg((const float4*)(a + (2 * h) * kHeadDim) + (j & 7));
  const float4 an = __ldg((const float4*)(a + (2 * h + 1) * kHeadDim) + (j & 7));
#pragma unroll
  for (int i = 0; i < NR; ++i) {
    *(float4*)&sm.Wh[R0 + i][4 * j] = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
    float s0 = as.x * acc[i][0] + as.y * acc[i][1] + as.z * acc[i][2] + as.w * acc[i][3];
    float s1 = an.x * acc[i][0] + an.y * acc[i][1] + an.z * acc[i][2] + an.w * acc[i][3];
#pragma unroll
    for (int o = 4; o >= 1; o >>= 1) {
      s0 += __shfl_xor_sync(0xffffffffu, s0, o);
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
    }
    if ((j & 7) == 0) {
      sm.ss[R0 + i][h] = s0;
      sm.sn[R0 + i][h] = s1;
    }
  }
}

// Rows R0..: sum over the stencil neighbours (ascending, as the CSR order)
// of alpha * Wh, + bias, ELU -> X.
template <int R0, int NR>
__device__ __forceinline__ void aggregate(const float* __restrict__ bias, TttSmem& sm, int j) {
  const int h = j >> 3;
  const float4 b4 = __ldg((const float4*)bias + j);
  const float bs[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
  for (int i = 0; i < NR; ++i) {
    const int r = R0 + i;
    float o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s = 0; s < kSlots; ++s) {
      const int nb = stencil(r, s);
      if (nb >= 0) {
        const float al = sm.alpha[r][s][h];
        const float4 x = *(const float4*)&sm.Wh[nb][4 * j];
        o[0] = fmaf(al, x.x, o[0]);
        o[1] = fmaf(al, x.y, o[1]);
        o[2] = fmaf(al, x.z, o[2]);
        o[3] = fmaf(al, x.w, o[3]);
      }
    }
    *(float4*)&sm.X[r][4 * j] = make_float4(elu(o[0] + bs[0]), elu(o[1] + bs[1]), elu(o[2] + bs[2]), elu(o[3] + bs[3]));
  }
}

__global__ void __launch_bounds__(kTT) gat_simt_ttt_kernel(const float* __restrict__ w, const int8_t* __restrict__ boards,
                                                           const int8_t* __restrict__ side_g, int n,
                                                           float* __restrict__ pi, float* __restrict__ v) {
  __shared__ __align__(16) TttSmem sm;
  const int t = threadIdx.x, j = t & 63, lane = t & 31;
  const bool first = t < 64;  // rows 0-4, else rows 5-8 (whole warps)
  const int gi = blockIdx.x;  // position (grid = n)
  const int side = side_g[gi];

  // encode: node r's four features in X[r][0..3]
  if (t < kN) {
    float f[TT::F];
    encode_node(kTicTacToe, boards + (size_t)gi * TT::BOARD, side, t, f);
    *(float4*)&sm.X[t][0] = make_float4(f[0], f[1], f[2], f[3]);
  }
  __syncthreads();

  for (int l = 0; l < TT::L; ++l) {
    const float* W = w + TttOff::W(l);
    {
      float acc[kHalf0][4];
#pragma unroll
      for (int i = 0; i < kHalf0; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
      if (first) {
        if (l == 0) project<0, kHalf0, TT::F>(W, sm, j, acc);
        else project<0, kHalf0, kHidden>(W, sm, j, acc);
        scores<0, kHalf0>(w + TttOff::a(l), sm, j, acc);
      } else {
        if (l == 0) project<kHalf0, kN - kHalf0, TT::F>(W, sm, j, acc);
        else project<kHalf0, kN - kHalf0, kHidden>(W, sm, j, acc);
        scores<kHalf0, kN - kHalf0>(w + TttOff::a(l), sm, j, acc);
      }
    }
    __syncthreads();
    // neighbour softmax per (node, head), weights by stencil slot
    if (t < kN * kHeads) {
      const int r = t >> 3, hh = t & 7;
      const float si = sm.ss[r][hh];
      float lg[kSlots];
      float m = -INFINITY;
#pragma unroll
      for (int s = 0; s < kSlots; ++s) {
        const int nb = stencil(r, s);
        lg[s] = nb >= 0 ? lrelu(si + sm.sn[nb < 0 ? 0 : nb][hh]) : -INFINITY;
        m = fmaxf(m, lg[s]);
      }
      float z = 0.f;
#pragma unroll
      for (int s = 0; s < kSlots; ++s) {
        const float p = stencil(r, s) >= 0 ? expf(lg[s] - m) : 0.f;
        lg[s] = p;
        z += p;
      }
      const float inv = 1.f / z;
#pragma unroll
      for (int s = 0; s < kSlots; ++s) sm.alpha[r][s][hh] = lg[s] * inv;
    }
    __syncthreads();
    if (first) aggregate<0, kHalf0>(w + TttOff::b(l), sm, j);
    else aggregate<kHalf0, kN - kHalf0>(w + TttOff::b(l), sm, j);
    __syncthreads();
  }

  // ---- heads ----
  // node mean (value head) and the per-node policy logit X_r . w_pi + b_pi,
  // the latter summed over the 64 column groups (warps 0 and 1)
  if (first) {
    const float4 wp = __ldg((const float4*)(w + TttOff::w_pi) + j);
    float lp[kN];
    float4 mean = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < kN; ++r) {
      const float4 x = *(const float4*)&sm.X[r][4 * j];
      mean.x += x.x;
      mean.y += x.y;
      mean.z += x.z;
      mean.w += x.w;
      lp[r] = x.x * wp.x + x.y * wp.y + x.z * wp.z + x.w * wp.w;
    }
    *(float4*)&sm.pooled[4 * j] =
        make_float4(mean.x * (1.0f / kN), mean.y * (1.0f / kN), mean.z * (1.0f / kN), mean.w * (1.0f / kN));
#pragma unroll
    for (int r = 0; r < kN; ++r) {
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) lp[r] += __shfl_xor_sync(0xffffffffu, lp[r], o);
    }
    if (lane == 0)
#pragma unroll
      for (int r = 0; r < kN; ++r) sm.red[t >> 5][r] = lp[r];
  }
  __syncthreads();
  // value hidden unit t: ReLU(b_v1 + pooled . W_v1[:, t]) in four partial sums
  if (first) {
    float a4[4] = {__ldg(w + TttOff::b_v1 + t), 0.f, 0.f, 0.f};
#pragma unroll 8
    for (int c = 0; c < kHidden; c += 4) {
      const float4 pc = *(const float4*)&sm.pooled[c];
      a4[0] = fmaf(pc.x, __ldg(w + TttOff::W_v1 + (size_t)c * kValueHidden + t), a4[0]);
      a4[1] = fmaf(pc.y, __ldg(w + TttOff::W_v1 + (size_t)(c + 1) * kValueHidden + t), a4[1]);
      a4[2] = fmaf(pc.z, __ldg(w + TttOff::W_v1 + (size_t)(c + 2) * kValueHidden + t), a4[2]);
      a4[3] = fmaf(pc.w, __ldg(w + TttOff::W_v1 + (size_t)(c + 3) * kValueHidden + t), a4[3]);
    }
    sm.hid[t] = fmaxf((a4[0] + a4[1]) + (a4[2] + a4[3]), 0.f);
  } else if (t - 64 < kN) {
    sm.logit[t - 64] = sm.red[0][t - 64] + sm.red[1][t - 64] + __ldg(w + TttOff::b_pi);
  }
  __syncthreads();
  // policy softmax over the 9 cells and the value output: warp 0
  if (t < 32) {
    const float lg = lane < kN ? sm.logit[lane] : -INFINITY;
    float m = lg;
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float e = lane < kN ? expf(lg - m) : 0.f;
    float z = e;
#pragma unroll
    for (int o = 16; o; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
    float vv = sm.hid[lane] * __ldg(w + TttOff::w_v2 + lane) + sm.hid[lane + 32] * __ldg(w + TttOff::w_v2 + lane + 32);
#pragma unroll
    for (int o = 16; o; o >>= 1) vv += __shfl_xor_sync(0xffffffffu, vv, o);
    if (gi < n) {
      if (lane < kN) pi[(size_t)gi * TT::A + lane] = e * (1.f / z);
      if (lane == 0) v[gi] = tanhf(vv + __ldg(w + TttOff::b_v2));
    }
  }
}

}  // namespace

// One CTA of 128 threads per position (n >= 1).
cudaError_t launch_gat_simt_ttt(const float* w, const int8_t* boards, const int8_t* side, int n, float* pi, float* v,
                                cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  gat_simt_ttt_kernel<<<n, kTT, 0, stream>>>(w, boards, side, n, pi, v);
  return cudaGetLastError();
}

}  // namespace gz
