// Connect4 ResNet training step: loss, backward pass and Adam, fp32 on CUDA
// cores, for the network the forward kernels evaluate (stem, 10 residual
// blocks with a real residual add, policy and value heads, BN in inference
// form).  The reference's losses are networks/resnet/resnet.cu:669-699; its
// backward_resnet (701-837) passes the input boards to every layer's filter
// gradient (796, 807), so it is not a gradient to reproduce: this computes
// the true one (checked against autograd in the tests).
//
// Convolutions are GEMMs over an im2col buffer: Z[rows][128] = col[rows][9 Cin]
// . W^T with W stored [Cout][ky][kx][Cin]; their backward passes are
// dW = dZ^T . col and dcol = dZ . W, folded back onto the input by a
// gather (col2im) that visits the taps in a fixed order.  BN is an affine
// map with fixed statistics: gamma and beta are trained, mean and variance
// get a zero gradient and are left alone by Adam.  The losses are those of
// the GAT training step (train.cu): softmax cross-entropy against pi plus
// the squared value error, averaged over the batch.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "gz_games.h"
#include "gz_internal.h"
#include "gz_train.h"

namespace gz {
namespace train {
namespace {

constexpr int kC = kResChannels;  // 128
constexpr int kNN = 42;           // squares
constexpr int kConvs = 1 + 2 * kResBlocks;

// Weight offsets of conv k (0 stem, 1 + 2 i and 2 + 2 i block i) and its BN.
size_t conv_w(const ResLayout& t, int k) { return k == 0 ? t.stem_w : (k % 2 ? t.conv1_w[(k - 1) / 2] : t.conv2_w[(k - 1) / 2]); }
size_t conv_bn(const ResLayout& t, int k) { return k == 0 ? t.stem_bn : (k % 2 ? t.bn1[(k - 1) / 2] : t.bn2[(k - 1) / 2]); }
int conv_cin(int k) { return k == 0 ? kResInPlanes : kC; }

// Arena parts (floats), for batches of up to B positions.
struct ResBuf {
  size_t x0;         // [rows][3] encoded input
  size_t A[kResBlocks + 1];  // block inputs a_0 (stem output) .. a_10, [rows][128]
  size_t T[kResBlocks];      // block intermediates t_i = ReLU(BN1(conv1(a_i)))
  size_t Z[kConvs];          // pre-BN conv outputs
  size_t col, dcol, dA, dT, dR, prod;
  size_t pz, vz, feat, vf, logits, h1, dlog, dh1, dvpre, terms, dfeat, dvf;
  size_t total;
};

ResBuf res_buf(int B) {
  const size_t rows = (size_t)B * kNN, act = rows * kC;
  ResBuf o{};
  size_t p = 0;
  auto take = [&](size_t n) {
    const size_t at = p;
    p += (n + 63) & ~(size_t)63;
    return at;
  };
  o.x0 = take(rows * kResInPlanes);
  for (auto& a : o.A) a = take(act);
  for (auto& t : o.T) t = take(act);
  for (auto& z : o.Z) z = take(act);
  o.col = take(rows * 9 * kC);
  o.dcol = take(rows * 9 * kC);
  o.dA = take(act);
  o.dT = take(act);
  o.dR = take(act);
  o.prod = take(act);
  o.pz = take(rows * 2);
  o.vz = take(rows);
  o.feat = take((size_t)B * 84);
  o.vf = take((size_t)B * kNN);
  o.logits = take((size_t)B * 7);
  o.h1 = take((size_t)B * kResValueHidden);
  o.dlog = take((size_t)B * 7);
  o.dh1 = take((size_t)B * kResValueHidden);
  o.dvpre = take(B);
  o.terms = take((size_t)B * 2);
  o.dfeat = take((size_t)B * 84);
  o.dvf = take((size_t)B * kNN);
  o.total = p;
  return o;
}

__global__ void res_encode_kernel(const int8_t* __restrict__ boards, const int8_t* __restrict__ side, int B,
                                  float* __restrict__ x0) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= B * kNN) return;
  const int b = r / kNN, sd = side[b], c = boards[r];
  x0[r * 3 + 0] = c == sd ? 1.f : 0.f;
  x0[r * 3 + 1] = c == -sd ? 1.f : 0.f;
  x0[r * 3 + 2] = sd == 1 ? 1.f : 0.f;
}

// col[row][(ky * 3 + kx) * cin + ci] = in[neighbour (ky - 1, kx - 1)][ci], 0 off the board
__global__ void im2col_kernel(const float* __restrict__ in, int cin, int rows, float* __restrict__ col) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x, K = (size_t)9 * cin;
  if (i >= (size_t)rows * K) return;
  const int row = (int)(i / K), j = (int)(i % K), tap = j / cin, ci = j % cin;
  const int p = row % kNN, r = p / 7 + tap / 3 - 1, c = p % 7 + tap % 3 - 1;
  col[i] = r >= 0 && r < 6 && c >= 0 && c < 7 ? in[(size_t)(row - p + r * 7 + c) * cin + ci] : 0.f;
}

// din[row][ci] = sum over taps (ascending) of dcol[the output row that read
// this one through the tap][tap * cin + ci]
__global__ void col2im_kernel(const float* __restrict__ dcol, int cin, int rows, float* __restrict__ din) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)rows * cin) return;
  const int row = (int)(i / cin), ci = (int)(i % cin), p = row % kNN;
  float acc = 0.f;
  for (int tap = 0; tap < 9; ++tap) {
    // output q read input p through tap: p = q + (tap / 3 - 1, tap % 3 - 1)
    const int r = p / 7 - (tap / 3 - 1), c = p % 7 - (tap % 3 - 1);
    if (r >= 0 && r < 6 && c >= 0 && c < 7) acc += dcol[(size_t)(row - p + r * 7 + c) * 9 * cin + tap * cin + ci];
  }
  din[i] = acc;
}

__device__ __forceinline__ float bn_inv(const float* bn, int C, int c) { return 1.f / sqrtf(bn[3 * C + c] + kBnEps); }

// out = ReLU(BN(z) [+ res]) over [rows][128]
__global__ void bn_relu_fwd_kernel(const float* __restrict__ z, const float* __restrict__ bn, const float* res,
                                   int rows, float* __restrict__ out) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)rows * kC) return;
  const int c = (int)(i % kC);
  float y = bn[c] * (z[i] - bn[2 * kC + c]) * bn_inv(bn, kC, c) + bn[kC + c];
  if (res) y += res[i];
  out[i] = fmaxf(y, 0.f);
}

// Backward of out = ReLU(BN(z) [+ res]) with BN's gradient sums: dpre =
// dout * (out > 0); dz = dpre * gamma * inv (dz may alias z); dres = dpre
// when given (the residual's gradient; may alias dout).  Block `slice` of
// kBnSlices takes a contiguous run of rows, thread c channel c, and writes
// the run's sums of dpre * xhat (gamma's gradient) and of dpre (beta's) to
// part[0][slice][c] and part[1][slice][c]; bn_sum_final_kernel adds the
// runs in order.
constexpr int kBnSlices = 256;
static_assert((size_t)2 * kBnSlices * kC <= kColsumFloats, "BN partial sums fit the column-sum scratch");
__global__ void __launch_bounds__(128) bn_relu_bwd_sum_kernel(const float* dout, const float* __restrict__ out,
                                                              const float* z, const float* __restrict__ bn, int rows,
                                                              float* dz, float* dres, float* __restrict__ part) {
  const int c = threadIdx.x, slice = blockIdx.x;
  const int per = (rows + kBnSlices - 1) / kBnSlices, r0 = slice * per, r1 = min(rows, r0 + per);
  const float inv = bn_inv(bn, kC, c), gamma = bn[c], mu = bn[2 * kC + c];
  float sg = 0.f, sb = 0.f;
  for (int r = r0; r < r1; ++r) {
    const size_t i = (size_t)r * kC + c;
    const float dpre = out[i] > 0.f ? dout[i] : 0.f;
    const float zi = z[i];
    dz[i] = dpre * gamma * inv;
    if (dres) dres[i] = dpre;
    sg = fmaf(dpre, (zi - mu) * inv, sg);
    sb += dpre;
  }
  part[slice * kC + c] = sg;
  part[(kBnSlices + slice) * kC + c] = sb;
}

// g_bn[0 .. 127] = gamma gradients, g_bn[128 .. 255] = beta gradients: one
// warp per output, lane l adding runs l, l + 32, ... in order, then a fixed
// shuffle tree over the lanes.
__global__ void __launch_bounds__(256) bn_sum_final_kernel(const float* __restrict__ part, float* __restrict__ g_bn) {
  const int o = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  const int which = o >> 7, c = o & 127;
  float s = 0.f;
  for (int k = lane; k < kBnSlices; k += 32) s += part[(which * kBnSlices + k) * kC + c];
#pragma unroll
  for (int w = 16; w >= 1; w >>= 1) s += __shfl_xor_sync(0xffffffffu, s, w);
  if (lane == 0) g_bn[which * kC + c] = s;
}

// The two 1x1 head convolutions and their BN, one warp per square:
// pz[row] = (pol_w[0] . a, pol_w[1] . a), vz[row] = val_w . a (pre-BN), and
// the BN outputs feat[b][o * 42 + pos] (policy) and vf[b][pos] (value).
__global__ void head_fwd_kernel(const float* __restrict__ a, const float* __restrict__ w, ResLayout t, int rows,
                                float* __restrict__ pz, float* __restrict__ vz, float* __restrict__ feat,
                                float* __restrict__ vf) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f;
  for (int c = lane; c < kC; c += 32) {
    const float x = a[(size_t)row * kC + c];
    s0 = fmaf(w[t.pol_w + c], x, s0);
    s1 = fmaf(w[t.pol_w + kC + c], x, s1);
    s2 = fmaf(w[t.val_w + c], x, s2);
  }
  for (int o = 16; o; o >>= 1) {
    s0 += __shfl_xor_sync(0xffffffffu, s0, o);
    s1 += __shfl_xor_sync(0xffffffffu, s1, o);
    s2 += __shfl_xor_sync(0xffffffffu, s2, o);
  }
  if (lane) return;
  const int b = row / kNN, pos = row % kNN;
  const float* pb = w + t.pol_bn;  // [4][2]
  const float* vb = w + t.val_bn;  // [4][1]
  pz[row * 2] = s0;
  pz[row * 2 + 1] = s1;
  vz[row] = s2;
  feat[(size_t)b * 84 + pos] = pb[0] * (s0 - pb[4]) * bn_inv(pb, 2, 0) + pb[2];
  feat[(size_t)b * 84 + kNN + pos] = pb[1] * (s1 - pb[5]) * bn_inv(pb, 2, 1) + pb[3];
  vf[(size_t)b * kNN + pos] = vb[0] * (s2 - vb[2]) * bn_inv(vb, 1, 0) + vb[1];
}

// Per position (128 threads): softmax cross-entropy of logits + fc bias
// against pi, the value h = ReLU(h1pre + b1), v = tanh(h . fc2 + b2), its
// squared error against z, and the gradients of loss / B: dlog (logits),
// dh1 (h1pre), dvpre (the tanh input); h is kept for fc2's gradient.
__global__ void __launch_bounds__(128) res_loss_kernel(const float* __restrict__ w, ResLayout t,
                                                       const float* __restrict__ logits, float* __restrict__ h1,
                                                       const float* __restrict__ pi, const float* __restrict__ vt,
                                                       float inv_batch, float* __restrict__ dlog,
                                                       float* __restrict__ dh1, float* __restrict__ dvpre,
                                                       float* __restrict__ terms) {
  __shared__ float red[4];
  const int b = blockIdx.x, u = threadIdx.x, lane = u & 31;
  // value head, one hidden unit per thread (h1 holds the pre-activation)
  const float pre = h1[(size_t)b * kResValueHidden + u] + w[t.val_fc1_b + u];
  const float h = fmaxf(pre, 0.f);
  float part = h * w[t.val_fc2 + u];
  for (int o = 16; o; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  if (lane == 0) red[u >> 5] = part;
  __syncthreads();
  const float vpre = ((red[0] + red[1]) + (red[2] + red[3])) + w[t.val_fc2_b];
  const float v = tanhf(vpre), z = vt[b];
  const float g = 2.f * (v - z) * (1.f - v * v) * inv_batch;
  h1[(size_t)b * kResValueHidden + u] = h;
  dh1[(size_t)b * kResValueHidden + u] = pre > 0.f ? g * w[t.val_fc2 + u] : 0.f;
  if (u >= 32) return;
  // policy: 7 logits on lanes 0..6
  const bool on = lane < 7;
  const float a = on ? logits[(size_t)b * 7 + lane] + w[t.pol_fc_b + lane] : -INFINITY;
  const float tp = on ? pi[(size_t)b * 7 + lane] : 0.f;
  float mx = a, se, st = tp;
  for (int o = 4; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  se = on ? expf(a - mx) : 0.f;
  for (int o = 4; o; o >>= 1) {
    se += __shfl_xor_sync(0xffffffffu, se, o);
    st += __shfl_xor_sync(0xffffffffu, st, o);
  }
  const float logz = mx + logf(se);
  float ce = on ? tp * (logz - a) : 0.f;
  for (int o = 4; o; o >>= 1) ce += __shfl_xor_sync(0xffffffffu, ce, o);
  if (on) dlog[(size_t)b * 7 + lane] = (expf(a - logz) * st - tp) * inv_batch;
  if (lane == 0) {
    dvpre[b] = g;
    terms[(size_t)b * 2] = ce;
    terms[(size_t)b * 2 + 1] = (z - v) * (z - v);
  }
}

// Backward of the head convolutions and their BN, one warp per square:
// dpz[row] = (policy 0, policy 1, value) gradients of the conv outputs,
// hb[row] = (dgamma_p0, dgamma_p1, dbeta_p0, dbeta_p1, dgamma_v, dbeta_v)
// terms, and da[row][c] = the three gradients through the 1x1 weights.
__global__ void head_bwd_kernel(const float* __restrict__ w, ResLayout t, const float* __restrict__ pz,
                                const float* __restrict__ vz, const float* __restrict__ dfeat,
                                const float* __restrict__ dvf, int rows, float* __restrict__ dpz,
                                float* __restrict__ hb, float* __restrict__ da) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int b = row / kNN, pos = row % kNN;
  const float* pb = w + t.pol_bn;
  const float* vb = w + t.val_bn;
  const float i0 = bn_inv(pb, 2, 0), i1 = bn_inv(pb, 2, 1), iv = bn_inv(vb, 1, 0);
  const float y0 = dfeat[(size_t)b * 84 + pos], y1 = dfeat[(size_t)b * 84 + kNN + pos], yv = dvf[(size_t)b * kNN + pos];
  const float d0 = y0 * pb[0] * i0, d1 = y1 * pb[1] * i1, dv = yv * vb[0] * iv;
  if (lane == 0) {
    dpz[row * 3] = d0;
    dpz[row * 3 + 1] = d1;
    dpz[row * 3 + 2] = dv;
    float* h = hb + (size_t)row * 6;
    h[0] = y0 * (pz[row * 2] - pb[4]) * i0;
    h[1] = y1 * (pz[row * 2 + 1] - pb[5]) * i1;
    h[2] = y0;
    h[3] = y1;
    h[4] = yv * (vz[row] - vb[2]) * iv;
    h[5] = yv;
  }
  for (int c = lane; c < kC; c += 32)
    da[(size_t)row * kC + c] = d0 * w[t.pol_w + c] + d1 * w[t.pol_w + kC + c] + dv * w[t.val_w + c];
}

// BN means and variances (fixed statistics) are not trained.
__device__ bool res_frozen(const ResLayout& t, size_t k) {
  const size_t C = kC, conv = C * 9 * C, block = 2 * (conv + 4 * C);
  if (k >= t.stem_bn && k < t.stem_bn + 4 * C) return k >= t.stem_bn + 2 * C;
  if (k >= t.conv1_w[0] && k < t.pol_w) {
    const size_t j = (k - t.conv1_w[0]) % block;
    return (j >= conv + 2 * C && j < conv + 4 * C) || j >= 2 * conv + 6 * C;
  }
  if (k >= t.pol_bn && k < t.pol_bn + 8) return k >= t.pol_bn + 4;
  if (k >= t.val_bn && k < t.val_bn + 4) return k >= t.val_bn + 2;
  return false;
}

// torch::optim::Adam as in train.cu's adam_kernel, skipping the BN statistics.
__global__ void res_adam_kernel(size_t n, ResLayout t, float* __restrict__ w, const float* __restrict__ grad,
                                float* __restrict__ m, float* __restrict__ v, AdamParams p, float bc1,
                                float bc2_sqrt) {
  const size_t k = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= n || res_frozen(t, k)) return;
  const float g = grad[k] * p.grad_scale + p.weight_decay * w[k];
  const float mk = p.beta1 * m[k] + (1.f - p.beta1) * g;
  const float vk = p.beta2 * v[k] + (1.f - p.beta2) * g * g;
  m[k] = mk;
  v[k] = vk;
  w[k] -= (p.lr / bc1) * mk / (sqrtf(vk) / bc2_sqrt + p.eps);
}

__global__ void add_kernel(size_t n, const float* __restrict__ a, float* __restrict__ acc) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) acc[i] += a[i];
}

unsigned blocks_for(size_t n, int threads) { return (unsigned)((n + threads - 1) / threads); }

}  // namespace

void res_bucket_range(int k, size_t* offset, size_t* count) {
  const ResLayout t = res_layout();
  if (k == 0) {  // heads
    *offset = t.pol_w;
    *count = t.total - t.pol_w;
  } else if (k <= kResBlocks) {  // block 10 - k (the backward pass meets the last block first)
    const int i = kResBlocks - k;
    *offset = t.conv1_w[i];
    *count = t.bn2[i] + 4 * kC - t.conv1_w[i];
  } else {  // stem
    *offset = t.stem_w;
    *count = t.conv1_w[0] - t.stem_w;
  }
}

cudaError_t res_ensure_state(State& st, int capacity) {
  cudaError_t e = cudaSuccess;
  if (st.kind != 1 || st.game != kConnect4) {
    free_state(st);
    st.kind = 1;
    st.game = kConnect4;
    st.weight_count = res_layout().total;
    const size_t wc = st.weight_count;
    if ((e = cudaMalloc(&st.m, wc * 4)) || (e = cudaMalloc(&st.v, wc * 4)) || (e = cudaMalloc(&st.grad, wc * 4)) ||
        (e = cudaMalloc(&st.loss, 2 * 4)))
      return e;
    // the BN statistics' gradient slots are never written: they stay 0
    if ((e = cudaMemset(st.m, 0, wc * 4)) || (e = cudaMemset(st.v, 0, wc * 4)) || (e = cudaMemset(st.grad, 0, wc * 4)))
      return e;
    st.ws.split_floats = (size_t)4 << 20;
    if ((e = cudaMalloc(&st.ws.split, st.ws.split_floats * 4)) || (e = cudaMalloc(&st.ws.colsum, kColsumFloats * 4)))
      return e;
    if ((e = cudaStreamCreateWithFlags(&st.comm_stream, cudaStreamNonBlocking))) return e;
    for (auto& ev : st.ev_bucket)
      if ((e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming))) return e;
    if ((e = cudaEventCreateWithFlags(&st.ev_comm, cudaEventDisableTiming))) return e;
  }
  if (capacity > st.capacity) {
    cudaFree(st.arena);
    st.arena = nullptr;
    st.capacity = 0;
    const ResBuf o = res_buf(capacity);
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

namespace {

// Backward of conv k's out = ReLU(BN(z) [+ res]) from dout: dz into `dz`
// (may be z), the residual's gradient into `dres` when given (may be dout),
// and the BN gamma and beta gradients into g.
cudaError_t bn_bwd(Workspace& ws, const ResLayout& t, int k, const float* w, const float* dout, const float* out,
                   const float* z, int rows, float* dz, float* dres, float* g, cudaStream_t s) {
  bn_relu_bwd_sum_kernel<<<kBnSlices, 128, 0, s>>>(dout, out, z, w + conv_bn(t, k), rows, dz, dres, ws.colsum);
  bn_sum_final_kernel<<<2 * kC / 8, 256, 0, s>>>(ws.colsum, g + conv_bn(t, k));
  return cudaGetLastError();
}

// conv k's weight gradient dW[Cout][9 Cin] = dz^T . im2col(in); with
// `din`, also din = col2im(dz . W) (+ `add` when given).  The 128-channel
// convolutions read im2col(in) in place; the 3-channel stem materialises it.
cudaError_t conv_bwd(Workspace& ws, const ResLayout& t, int k, const float* w, const float* in, const float* dz,
                     float* col, float* dcol, int rows, float* g, float* din, const float* add, cudaStream_t s) {
  const int cin = conv_cin(k), K = 9 * cin;
  if (cin == kC && gemm_big(kC, K)) {
    GZ_TRY(gemm(ws, kC, K, rows, dz, kC, true, in, 0, false, g + conv_w(t, k), K, false, s, 2));
  } else {
    im2col_kernel<<<blocks_for((size_t)rows * K, 256), 256, 0, s>>>(in, cin, rows, col);
    GZ_TRY(gemm(ws, kC, K, rows, dz, kC, true, col, K, false, g + conv_w(t, k), K, false, s));
  }
  if (!din) return cudaGetLastError();
  GZ_TRY(gemm(ws, rows, K, kC, dz, kC, false, w + conv_w(t, k), K, false, dcol, K, false, s));
  col2im_kernel<<<blocks_for((size_t)rows * cin, 256), 256, 0, s>>>(dcol, cin, rows, din);
  if (add) add_kernel<<<blocks_for((size_t)rows * cin, 256), 256, 0, s>>>((size_t)rows * cin, add, din);
  return cudaGetLastError();
}

// Z = im2col(in) . W^T for conv k (in place for 128 channels, as conv_bwd)
cudaError_t conv_fwd(Workspace& ws, const ResLayout& t, int k, const float* w, const float* in, float* col,
                     float* z, int rows, cudaStream_t s) {
  const int cin = conv_cin(k), K = 9 * cin;
  if (cin == kC && gemm_big(rows, kC)) return gemm(ws, rows, kC, K, in, 0, false, w + conv_w(t, k), K, true, z, kC, false, s, 1);
  im2col_kernel<<<blocks_for((size_t)rows * K, 256), 256, 0, s>>>(in, cin, rows, col);
  return gemm(ws, rows, kC, K, col, K, false, w + conv_w(t, k), K, true, z, kC, false, s);
}

}  // namespace

cudaError_t res_loss_and_grad(State& st, const float* w, const int8_t* boards, const int8_t* side, const float* pi,
                              const float* v, int B, cudaStream_t s,
                              const std::function<cudaError_t(int)>& bucket_done) {
  if (B <= 0 || B > st.capacity || st.kind != 1) return cudaErrorInvalidValue;
  const ResLayout t = res_layout();
  const ResBuf o = res_buf(st.capacity);
  const int rows = B * kNN;
  const size_t act = (size_t)rows * kC;
  float* ar = st.arena;
  float* g = st.grad;
  Workspace& ws = st.ws;
  float* col = ar + o.col;
  float* dcol = ar + o.dcol;

  // ---- forward ----
  res_encode_kernel<<<blocks_for(rows, 256), 256, 0, s>>>(boards, side, B, ar + o.x0);
  GZ_TRY(conv_fwd(ws, t, 0, w, ar + o.x0, col, ar + o.Z[0], rows, s));
  bn_relu_fwd_kernel<<<blocks_for(act, 256), 256, 0, s>>>(ar + o.Z[0], w + t.stem_bn, nullptr, rows, ar + o.A[0]);
  for (int i = 0; i < kResBlocks; ++i) {
    GZ_TRY(conv_fwd(ws, t, 1 + 2 * i, w, ar + o.A[i], col, ar + o.Z[1 + 2 * i], rows, s));
    bn_relu_fwd_kernel<<<blocks_for(act, 256), 256, 0, s>>>(ar + o.Z[1 + 2 * i], w + t.bn1[i], nullptr, rows,
                                                           ar + o.T[i]);
    GZ_TRY(conv_fwd(ws, t, 2 + 2 * i, w, ar + o.T[i], col, ar + o.Z[2 + 2 * i], rows, s));
    bn_relu_fwd_kernel<<<blocks_for(act, 256), 256, 0, s>>>(ar + o.Z[2 + 2 * i], w + t.bn2[i], ar + o.A[i], rows,
                                                           ar + o.A[i + 1]);
  }
  const float* top = ar + o.A[kResBlocks];
  head_fwd_kernel<<<blocks_for(rows, 8), 256, 0, s>>>(top, w, t, rows, ar + o.pz, ar + o.vz, ar + o.feat, ar + o.vf);
  GZ_TRY(gemm(ws, B, 7, 84, ar + o.feat, 84, false, w + t.pol_fc, 7, false, ar + o.logits, 7, false, s));
  GZ_TRY(gemm(ws, B, kResValueHidden, kNN, ar + o.vf, kNN, false, w + t.val_fc1, kResValueHidden, false, ar + o.h1,
              kResValueHidden, false, s));
  res_loss_kernel<<<B, 128, 0, s>>>(w, t, ar + o.logits, ar + o.h1, pi, v, 1.f / (float)B, ar + o.dlog, ar + o.dh1,
                                    ar + o.dvpre, ar + o.terms);
  GZ_TRY(colsum(ws, ar + o.terms, B, 2, 2, st.loss, false, s, 1.f / (float)B));

  // ---- heads backward ----
  GZ_TRY(gemm(ws, kResValueHidden, 1, B, ar + o.h1, kResValueHidden, true, ar + o.dvpre, 1, false, g + t.val_fc2, 1,
              false, s));
  GZ_TRY(colsum(ws, ar + o.dvpre, B, 1, 1, g + t.val_fc2_b, false, s));
  GZ_TRY(gemm(ws, kNN, kResValueHidden, B, ar + o.vf, kNN, true, ar + o.dh1, kResValueHidden, false, g + t.val_fc1,
              kResValueHidden, false, s));
  GZ_TRY(colsum(ws, ar + o.dh1, B, kResValueHidden, kResValueHidden, g + t.val_fc1_b, false, s));
  GZ_TRY(gemm(ws, 84, 7, B, ar + o.feat, 84, true, ar + o.dlog, 7, false, g + t.pol_fc, 7, false, s));
  GZ_TRY(colsum(ws, ar + o.dlog, B, 7, 7, g + t.pol_fc_b, false, s));
  GZ_TRY(gemm(ws, B, kNN, kResValueHidden, ar + o.dh1, kResValueHidden, false, w + t.val_fc1, kResValueHidden, true,
              ar + o.dvf, kNN, false, s));
  GZ_TRY(gemm(ws, B, 84, 7, ar + o.dlog, 7, false, w + t.pol_fc, 7, true, ar + o.dfeat, 84, false, s));
  // dpz [rows][3] and the six BN terms [rows][6] share the prod buffer
  float* dpz = ar + o.prod;
  float* hb = dpz + (size_t)rows * 3;
  float* dA = ar + o.dA;
  head_bwd_kernel<<<blocks_for(rows, 8), 256, 0, s>>>(w, t, ar + o.pz, ar + o.vz, ar + o.dfeat, ar + o.dvf, rows, dpz,
                                                     hb, dA);
  GZ_TRY(gemm(ws, 2, kC, rows, dpz, 3, true, top, kC, false, g + t.pol_w, kC, false, s));
  GZ_TRY(gemm(ws, 1, kC, rows, dpz + 2, 3, true, top, kC, false, g + t.val_w, kC, false, s));
  GZ_TRY(colsum(ws, hb, rows, 4, 6, g + t.pol_bn, false, s));
  GZ_TRY(colsum(ws, hb + 4, rows, 2, 6, g + t.val_bn, false, s));
  GZ_TRY(cudaGetLastError());
  GZ_TRY(bucket_done(0));

  // ---- residual blocks backward, last first ----
  // Each conv's output gradient overwrites its saved pre-BN output Z[k],
  // which the backward pass no longer needs once BN's backward has read it.
  float* dR = ar + o.dR;  // gradient of the block input through the residual add
  float* dT = ar + o.dT;
  for (int i = kResBlocks - 1; i >= 0; --i) {
    const int k1 = 1 + 2 * i, k2 = 2 + 2 * i;
    // a_{i+1} = ReLU(BN2(z2) + a_i)
    GZ_TRY(bn_bwd(ws, t, k2, w, dA, ar + o.A[i + 1], ar + o.Z[k2], rows, ar + o.Z[k2], dR, g, s));
    // z2 = conv2(t_i): Z[k2] now holds dz2
    GZ_TRY(conv_bwd(ws, t, k2, w, ar + o.T[i], ar + o.Z[k2], col, dcol, rows, g, dT, nullptr, s));
    // t_i = ReLU(BN1(z1))
    GZ_TRY(bn_bwd(ws, t, k1, w, dT, ar + o.T[i], ar + o.Z[k1], rows, ar + o.Z[k1], nullptr, g, s));
    // z1 = conv1(a_i); da_i = dR + col2im(dz1 . W1)
    GZ_TRY(conv_bwd(ws, t, k1, w, ar + o.A[i], ar + o.Z[k1], col, dcol, rows, g, dA, dR, s));
    GZ_TRY(bucket_done(kResBlocks - i));
  }
  // ---- stem ----
  GZ_TRY(bn_bwd(ws, t, 0, w, dA, ar + o.A[0], ar + o.Z[0], rows, ar + o.Z[0], nullptr, g, s));
  GZ_TRY(conv_bwd(ws, t, 0, w, ar + o.x0, ar + o.Z[0], col, dcol, rows, g, nullptr, nullptr, s));
  GZ_TRY(bucket_done(kResBlocks + 1));
  return cudaSuccess;
}

cudaError_t res_adam_step(State& st, float* w, const AdamParams& p, cudaStream_t s) {
  st.step += 1;
  const double bc1 = 1.0 - pow((double)p.beta1, (double)st.step);
  const double bc2 = 1.0 - pow((double)p.beta2, (double)st.step);
  const size_t n = st.weight_count;
  res_adam_kernel<<<blocks_for(n, 256), 256, 0, s>>>(n, res_layout(), w, st.grad, st.m, st.v, p, (float)bc1,
                                                     (float)sqrt(bc2));
  return cudaGetLastError();
}

}  // namespace train
}  // namespace gz
