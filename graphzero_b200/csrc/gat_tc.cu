// Tensor-core (tcgen05) GAT forward for Connect4: all six layers and both
// heads in one persistent launch, one CTA per SM.
//
// A tile is 128 node rows = 3 positions x 42 nodes (+2 padding rows).  Per
// layer:
//   1. projection   Wh[128 x 256] = X[128 x K] . W[K x 256]       (tcgen05.mma,
//      bf16/fp16 operands from shared memory, fp32 accumulator in tensor
//      memory: lane = node, column = feature)
//   2. per head h (8 heads, two groups of four run by two warpgroups):
//      scores   s_i = a_self . Wh_i^h, t_i = a_nbr . Wh_i^h      (in-thread)
//      softmax  alpha_ij = softmax_j LeakyReLU_0.2(s_i + t_j) over the
//               8-neighbourhood + self of node i (the Connect4 board graph)
//      gather   out^h = alpha^h . Wh^h   as a second tcgen05.mma: alpha^h
//               (128 x 128, fp16, block-diagonal, zero outside each node's
//               3x3 stencil) is the A operand in tensor memory, Wh^h (fp16)
//               the B operand in shared memory; the result overwrites the
//               head's accumulator columns
//   3. bias + ELU, stored as the next layer's X tile (128-byte swizzled,
//      K-major) -- or, after the last layer, mean-pooled into the value head
//      (256->64 ReLU, 64->1 tanh) and column-pooled into the policy head
//      (256->1 per column, softmax over 7), in fp32.
// Weights W_l^T are pre-packed on the device into 32 KB chunks (256 feature
// rows x 64 K, swizzled) and streamed into a two-slot shared-memory ring by
// one producer thread with 1-D bulk async copies (TMA engine); one thread
// issues every MMA.  Every wait is bounded (%globaltimer); on a timeout the
// CTA drains its copies and MMAs, frees tensor memory and reports through
// the error word.
//
// Reference: networks/gat/gat.cu:836-870 (forward_gat_layer), 916-948
// (compute_output), 995-1038 (softmax, tanh); the math is the standard GAT
// the reference's kernels never completed.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "gz_games.h"
#include "gz_internal.h"
#include "gz_sm100.h"

namespace gz {
namespace {

using namespace sm100;

constexpr int kN = 42;              // Connect4 nodes
constexpr int kGPT = 3;             // positions per tile
constexpr int kRows = 128;          // MMA M (node rows per tile)
constexpr int kLayers = 6;
constexpr int kEpiWarps = 8;        // two warpgroups: heads 0-3 and 4-7
constexpr int kThreads = (kEpiWarps + 2) * 32;
constexpr int kProducerWarp = kEpiWarps;
constexpr int kMmaWarp = kEpiWarps + 1;
constexpr int kWChunk = 32768;      // 256 feature rows x 64 K x 2 B
constexpr int kWSlots = 2;
constexpr int kChunksPerTile = 1 + (kLayers - 1) * 4;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kAlphaCol = 256;  // alpha buffers: 256 + (2 * group + buffer) * 64
constexpr uint64_t kWaitLimitNs = 4000000000ull;  // 4 s per wait

// Shared memory map (bytes).
constexpr int kSmX = 0;                                // X tile: 4 x 16 KB (K-major, 128 rows)
constexpr int kSmW = kSmX + 4 * 16384;                 // weight ring
constexpr int kSmB2 = kSmW + kWSlots * kWChunk;        // Wh^h operand: [group][buffer] 8 KB each
constexpr int kSmStage = kSmB2 + 4 * 8192;             // alpha staging: [group][24 words][128 nodes]
constexpr int kSmScore = kSmStage + 2 * 24 * 128 * 4;  // [group][buffer][128][2] floats
constexpr int kSmVec = kSmScore + 2 * 2 * 128 * 2 * 4; // per layer: a[8][2][32], bias[256]; x2 (layer parity)
constexpr int kVecFloats = 8 * 2 * 32 + 256;
constexpr int kSmBar = kSmVec + 2 * kVecFloats * 4;
constexpr int kNumBars = 2 * kWSlots + 1 + 1 + 4 + 4 + 1;  // full, empty, acc_full, x_ready, req[2][2], done2[2][2], drain
constexpr int kSmMisc = kSmBar + kNumBars * 8;
constexpr int kSmemBytes = kSmMisc + 16;
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
// last-layer head scratch inside the (then unused) X tile
constexpr int kHeadRowStride = 33;                      // floats, padded
constexpr int kSmHeadRows = kSmX;                       // [group][128][33] floats
constexpr int kSmPooled = kSmHeadRows + 2 * 128 * kHeadRowStride * 4;  // [3][256]
constexpr int kSmPcol = kSmPooled + kGPT * 256 * 4;     // [3][7][256] column means
constexpr int kSmZ = kSmPcol + kGPT * 7 * 256 * 4;      // [3][64]
constexpr int kSmLogit = kSmZ + kGPT * 64 * 4;          // [3][8]
static_assert(kSmLogit + kGPT * 8 * 4 <= kSmW, "head scratch fits in the X tile");

// Offsets (floats) into the fp32 weight blob for Connect4 (gat_layout order).
struct C4Off {
  static constexpr int kLayer0 = 4 * 256 + 256 + 512;
  static constexpr int kLayerN = 256 * 256 + 256 + 512;
  __device__ static constexpr int W(int l) { return l == 0 ? 0 : kLayer0 + (l - 1) * kLayerN; }
  __device__ static constexpr int b(int l) { return W(l) + (l == 0 ? 4 : 256) * 256; }
  __device__ static constexpr int a(int l) { return b(l) + 256; }
  static constexpr int kHeads = kLayer0 + (kLayers - 1) * kLayerN;
  static constexpr int w_pi = kHeads, b_pi = w_pi + 256, W_v1 = b_pi + 1, b_v1 = W_v1 + 256 * 64;
  static constexpr int w_v2 = b_v1 + 64, b_v2 = w_v2 + 64;
};

template <typename T> struct OpType;
template <> struct OpType<__nv_bfloat16> {
  static constexpr uint32_t fmt = 1;
  static __device__ __forceinline__ uint16_t bits(float x) { return __bfloat16_as_ushort(__float2bfloat16_rn(x)); }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};
template <> struct OpType<__half> {
  static constexpr uint32_t fmt = 0;
  static __device__ __forceinline__ uint16_t bits(float x) { return __half_as_ushort(__float2half_rn(x)); }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Barrier over the epilogue warps that also ANDs `ok` across them, so they
// continue or give up together (no warp is left behind in a later barrier).
__device__ __forceinline__ bool epilogue_all(bool ok) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 2, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)ok), "r"(kEpiWarps * 32)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ float lrelu(float x) { return x > 0.f ? x : kLeakySlope * x; }
__device__ __forceinline__ float elu_fast(float x) { return x > 0.f ? x : __expf(x) - 1.0f; }

// First node of the 48-node window that covers every neighbour of the 32
// nodes owned by lane quarter q (nodes 32q .. 32q+31 have neighbours within
// +-8); clamped to [0, 80] so the window stays inside the 128 columns.
__device__ __forceinline__ int window_start(int q) { return q == 0 ? 0 : q == 3 ? 80 : 32 * q - 8; }

struct TcParams {
  const uint8_t* packed;  // kChunksPerTile chunks in consumption order
  const float* w;         // fp32 blob (biases, attention vectors, heads)
  const int8_t* boards;
  const int8_t* side;
  float* pi;
  float* v;
  int* err;
  int n;
  int num_tiles;
};

template <typename OpT>
__global__ void __launch_bounds__(kThreads, 1) gat_tc_c4_kernel(TcParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  if (smem_u32(smem) & 1023u) {  // swizzled operand tiles need a 1024-byte aligned base
    if (threadIdx.x == 0) atomicExch(p.err, 2);
    return;
  }
  uint8_t* sX = smem + kSmX;
  uint8_t* sW = smem + kSmW;
  uint64_t* bars = (uint64_t*)(smem + kSmBar);
  uint64_t* full = bars;
  uint64_t* empty = bars + kWSlots;
  uint64_t* acc_full = bars + 2 * kWSlots;
  uint64_t* x_ready = acc_full + 1;
  // req / done2 per (group, buffer): a head's gather request and its
  // completion.  One barrier per buffer keeps every producer at most one
  // phase ahead of its consumer.
  uint64_t* req = acc_full + 2;     // [2 groups][2 buffers]
  uint64_t* done2 = acc_full + 6;   // [2 groups][2 buffers]
  uint64_t* drain = acc_full + 10;
  uint32_t* tmem_slot = (uint32_t*)(smem + kSmMisc);
  volatile int* abort_flag = (volatile int*)(smem + kSmMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // zero the alpha staging (its zero pattern is static) and init barriers
  for (int i = threadIdx.x; i < 2 * 24 * 128; i += blockDim.x) ((uint32_t*)(smem + kSmStage))[i] = 0u;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kWSlots; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(x_ready, kEpiWarps);
    for (int i = 0; i < 4; ++i) {
      mbar_init(&req[i], 4);
      mbar_init(&done2[i], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kProducerWarp) {
    // ---------------- weight producer ----------------
    if (lane == 0) {
      uint32_t q = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        for (int c = 0; c < kChunksPerTile && ok; ++c, ++q) {
          const int s = q % kWSlots;
          ok = mbar_wait(&empty[s], ((q / kWSlots) & 1) ^ 1, abort_flag, kWaitLimitNs);
          if (!ok) break;
          mbar_arrive_expect_tx(&full[s], kWChunk);
          bulk_g2s(sW + s * kWChunk, p.packed + (size_t)c * kWChunk, kWChunk, &full[s]);
        }
      }
      for (uint32_t k = (q > kWSlots ? q - kWSlots : 0); k < q; ++k)  // every issued copy lands
        mbar_wait(&full[k % kWSlots], (k / kWSlots) & 1, abort_flag, kWaitLimitNs);
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc1 = idesc_f16(OpType<OpT>::fmt, 128, 256);
      constexpr uint32_t idesc2 = idesc_f16(0 /* fp16 */, 128, 32, 1 /* B N-contiguous */);
      const uint32_t xs = smem_u32(sX);
      const uint32_t b2s = smem_u32(smem + kSmB2);
      uint32_t q = 0, xph = 0, rph[4] = {0, 0, 0, 0};
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        for (int l = 0; l < kLayers && ok; ++l) {
          ok = mbar_wait(x_ready, xph & 1, abort_flag, kWaitLimitNs);
          ++xph;
          if (!ok) break;
          tc_fence_after();
          const int nchunk = l == 0 ? 1 : 4;  // K chunks of 64
          const int ksteps = l == 0 ? 1 : 4;  // K = 16 per MMA (layer 0: 4 features -> one step)
          for (int c = 0; c < nchunk && ok; ++c, ++q) {
            const int s = q % kWSlots;
            ok = mbar_wait(&full[s], (q / kWSlots) & 1, abort_flag, kWaitLimitNs);
            if (!ok) break;
            tc_fence_after();
            const uint32_t ws = smem_u32(sW + s * kWChunk);
            for (int kk = 0; kk < ksteps; ++kk)
              mma_f16_ss(tmem, sw128_desc(xs + c * 16384 + kk * 32), sw128_desc(ws + kk * 32), idesc1, (c | kk) != 0);
            mma_commit(&empty[s]);
          }
          if (!ok) break;
          mma_commit(acc_full);
          // gathers: serve whichever group's next head is ready (each group's
          // heads in order), eight per layer
          int next_t[2] = {0, 0};
          uint64_t t0 = global_timer_ns();
          while (ok && (next_t[0] < 4 || next_t[1] < 4)) {
            bool issued = false;
            for (int g = 0; g < 2; ++g) {
              if (next_t[g] >= 4) continue;
              const int t = next_t[g], b = t & 1, h = 4 * g + t;
              if (!mbar_try_wait(&req[2 * g + b], rph[2 * g + b] & 1)) continue;
              ++rph[2 * g + b];
              ++next_t[g];
              tc_fence_after();
              const uint32_t a_col = tmem + kAlphaCol + (uint32_t)((2 * g + b) * 64);
              const uint32_t bb = b2s + (uint32_t)((2 * g + b) * 8192);
              for (int kk = 0; kk < 8; ++kk)  // K = 16 nodes = two 8-row core-matrix groups per step
                mma_f16_ts(tmem + (uint32_t)(32 * h), a_col + kk * 8, noswizzle_desc(bb + kk * 1024, 512, 128), idesc2,
                           kk != 0);
              mma_commit(&done2[2 * g + b]);
              issued = true;
            }
            if (issued) {
              t0 = global_timer_ns();
            } else if (*abort_flag || global_timer_ns() - t0 > kWaitLimitNs) {
              *abort_flag = 1;
              ok = false;
            }
          }
        }
      }
      mma_commit(drain);
      mbar_wait(drain, 0, abort_flag, kWaitLimitNs);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue: warpgroup g owns heads 4g..4g+3 ----------------
    const int g = warp >> 2, qd = warp & 3;
    const int i = 32 * qd + lane;  // node row of this thread
    const uint32_t tlane = tmem + ((uint32_t)(32 * qd) << 16);
    const int li = i % kN, rr = li / 7, cc = li % 7;
    const bool real = i < kGPT * kN;
    const int jw0 = window_start(qd);
    uint32_t* stage = (uint32_t*)(smem + kSmStage) + g * 24 * 128;
    // node i's 3x3 stencil: validity bits and the staging address of each
    // neighbour's alpha (word (j - jw0) / 2 of column i, half (j - jw0) % 2)
    uint32_t nmask = 0, saddr[9];
#pragma unroll
    for (int k = 0; k < 9; ++k) {
      const int dr = k / 3 - 1, dc = k % 3 - 1;
      const bool in = real && (unsigned)(rr + dr) < 6u && (unsigned)(cc + dc) < 7u;
      nmask |= (uint32_t)in << k;
      const int wpos = in ? i + 7 * dr + dc - jw0 : 0;  // 0..47
      saddr[k] = smem_u32(stage + (wpos >> 1) * 128 + i) + (wpos & 1) * 2;
    }
    float* score = (float*)(smem + kSmScore) + g * 2 * 128 * 2;
    const int gbar = 3 + g;
    uint32_t aph = 0, dph[2] = {0, 0};
    bool ok = true;

    // zero this warp's lanes of both alpha buffers of its group (static background)
    {
      uint32_t z[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int b = 0; b < 2; ++b)
        for (int c = 0; c < 64; c += 8) tmem_st_x8(tlane + kAlphaCol + (2 * g + b) * 64 + c, z);
      tmem_st_wait();
    }

    for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
      // -- encode the tile's positions into X chunk 0 (features 0..15) --
      for (int t = threadIdx.x; t < kRows * 2; t += kEpiWarps * 32) {
        const int j = t >> 1, half = t & 1;
        const int gj = j / kN, lj = j % kN;
        const int pos = tile * kGPT + gj;
        uint32_t wv[4] = {0, 0, 0, 0};
        if (half == 0 && gj < kGPT && pos < p.n) {
          float f[4];
          encode_node(kConnect4, p.boards + (size_t)pos * 42, p.side[pos], lj, f);
          wv[0] = OpType<OpT>::pack(f[0], f[1]);
          wv[1] = OpType<OpT>::pack(f[2], f[3]);
        }
        *(uint4*)(sX + sw128_offset(j, half * 8)) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(x_ready);

      for (int l = 0; l < kLayers && ok; ++l) {
        const bool last = l == kLayers - 1;
        // per-layer vectors (attention a, bias) into shared memory, by layer parity
        float* vec = (float*)(smem + kSmVec) + (l & 1) * kVecFloats;
        for (int t = threadIdx.x; t < kVecFloats; t += kEpiWarps * 32)
          vec[t] = t < 512 ? __ldg(p.w + C4Off::a(l) + t) : __ldg(p.w + C4Off::b(l) + t - 512);
        ok = epilogue_all(mbar_wait(acc_full, aph & 1, abort_flag, kWaitLimitNs));  // also publishes vec
        ++aph;
        if (!ok) break;
        tc_fence_after();

        float* hrow = (float*)(smem + kSmHeadRows) + g * 128 * kHeadRowStride;
        float* pcol = (float*)(smem + kSmPcol);
        float* pooled = (float*)(smem + kSmPooled);

        // P3: result of head t -> bias, ELU -> next X (or head pooling)
        auto finish_head = [&](int t) {
          const int h = 4 * g + t, b = t & 1;
          ok = mbar_wait(&done2[2 * g + b], dph[b] & 1, abort_flag, kWaitLimitNs) && ok;
          ++dph[b];
          tc_fence_after();
          float o[32];
          tmem_ld_x32(tlane + (uint32_t)(32 * h), o);
          tmem_ld_wait();
          const float4* bias4 = (const float4*)(vec + 512 + 32 * h);
          if (!last) {
            uint32_t w[16];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const float4 bv = bias4[k];
              w[2 * k] = OpType<OpT>::pack(elu_fast(o[4 * k] + bv.x), elu_fast(o[4 * k + 1] + bv.y));
              w[2 * k + 1] = OpType<OpT>::pack(elu_fast(o[4 * k + 2] + bv.z), elu_fast(o[4 * k + 3] + bv.w));
            }
            uint8_t* xrow = sX + (h >> 1) * 16384 + (i >> 3) * 1024 + (i & 7) * 128;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int unit = (4 * (h & 1) + u) ^ (i & 7);
              *(uint4*)(xrow + unit * 16) = make_uint4(w[4 * u], w[4 * u + 1], w[4 * u + 2], w[4 * u + 3]);
            }
          } else {
            // fp32 rows of this head into scratch, then per-position pooling
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const float4 bv = bias4[k];
              hrow[i * kHeadRowStride + 4 * k + 0] = elu_fast(o[4 * k + 0] + bv.x);
              hrow[i * kHeadRowStride + 4 * k + 1] = elu_fast(o[4 * k + 1] + bv.y);
              hrow[i * kHeadRowStride + 4 * k + 2] = elu_fast(o[4 * k + 2] + bv.z);
              hrow[i * kHeadRowStride + 4 * k + 3] = elu_fast(o[4 * k + 3] + bv.w);
            }
            named_bar_sync(gbar, 128);
            const int tid = threadIdx.x & 127;
            if (tid < kGPT * 32) {
              const int pg = tid >> 5, d = tid & 31;
              float cs[7] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, tot = 0.f;
#pragma unroll
              for (int r = 0; r < 6; ++r)
#pragma unroll
                for (int c = 0; c < 7; ++c) {
                  const float x = hrow[(pg * kN + r * 7 + c) * kHeadRowStride + d];
                  cs[c] += x;
                  tot += x;
                }
              pooled[pg * 256 + 32 * h + d] = tot * (1.0f / kN);
#pragma unroll
              for (int c = 0; c < 7; ++c) pcol[(pg * 7 + c) * 256 + 32 * h + d] = cs[c] * (1.0f / 6.0f);
            }
            named_bar_sync(gbar, 128);  // scratch reused by the next head
          }
        };

        // The head loop always runs to the end (waits return at once after an
        // abort), so every thread meets every named barrier; the decision to
        // stop is collective, at the end of the layer.
        for (int t = 0; t < 4; ++t) {
          const int h = 4 * g + t, b = t & 1;
          // ---- P1: Wh^h (fp32) -> scores, fp16 copy as the gather's B operand ----
          float wh[32];
          tmem_ld_x32(tlane + (uint32_t)(32 * h), wh);
          tmem_ld_wait();
          const float4* as4 = (const float4*)(vec + (h * 2 + 0) * 32);
          const float4* an4 = (const float4*)(vec + (h * 2 + 1) * 32);
          // four independent partial sums per score (short dependency chains)
          float sp[4] = {0.f, 0.f, 0.f, 0.f}, tp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const float4 a1 = as4[k], a2 = an4[k];
            sp[0] = fmaf(a1.x, wh[4 * k], sp[0]); sp[1] = fmaf(a1.y, wh[4 * k + 1], sp[1]);
            sp[2] = fmaf(a1.z, wh[4 * k + 2], sp[2]); sp[3] = fmaf(a1.w, wh[4 * k + 3], sp[3]);
            tp[0] = fmaf(a2.x, wh[4 * k], tp[0]); tp[1] = fmaf(a2.y, wh[4 * k + 1], tp[1]);
            tp[2] = fmaf(a2.z, wh[4 * k + 2], tp[2]); tp[3] = fmaf(a2.w, wh[4 * k + 3], tp[3]);
          }
          const float si = (sp[0] + sp[1]) + (sp[2] + sp[3]);
          const float ti = (tp[0] + tp[1]) + (tp[2] + tp[3]);
          // Wh^h (fp16) as the gather's B operand, N-contiguous without swizzle:
          // node i's 8-feature group ng at ng * 128 + (i / 8) * 512 + (i % 8) * 16
          {
            uint8_t* b2 = smem + kSmB2 + (2 * g + b) * 8192 + (i >> 3) * 512 + (i & 7) * 16;
#pragma unroll
            for (int ng = 0; ng < 4; ++ng)
              *(uint4*)(b2 + ng * 128) =
                  make_uint4(OpType<__half>::pack(wh[8 * ng + 0], wh[8 * ng + 1]), OpType<__half>::pack(wh[8 * ng + 2], wh[8 * ng + 3]),
                             OpType<__half>::pack(wh[8 * ng + 4], wh[8 * ng + 5]), OpType<__half>::pack(wh[8 * ng + 6], wh[8 * ng + 7]));
          }
          ((float2*)score)[b * 128 + i] = make_float2(si, ti);
          fence_proxy_async_smem();
          tc_fence_before();
          named_bar_sync(gbar, 128);  // scores of every node of the head are visible
          // ---- P2: neighbour softmax of node i -> alpha row (fp16) in tensor memory ----
          {
            const float2* sc = (const float2*)score + b * 128;
            float ev[9];
            float mx = -INFINITY;
#pragma unroll
            for (int k = 0; k < 9; ++k) {
              const int dr = k / 3 - 1, dc = k % 3 - 1;
              ev[k] = (nmask >> k) & 1u ? lrelu(si + sc[i + 7 * dr + dc].y) : -INFINITY;
              mx = fmaxf(mx, ev[k]);
            }
            float z = 0.f;
#pragma unroll
            for (int k = 0; k < 9; ++k) {
              ev[k] = ev[k] == -INFINITY ? 0.f : __expf(ev[k] - mx);
              z += ev[k];
            }
            const float inv = real ? 1.0f / z : 0.f;
#pragma unroll
            for (int k = 0; k < 9; ++k)
              if ((nmask >> k) & 1u)
                asm volatile("st.shared.b16 [%0], %1;" ::"r"(saddr[k]), "h"(OpType<__half>::bits(ev[k] * inv)) : "memory");
            uint32_t a[24];
#pragma unroll
            for (int k = 0; k < 24; ++k) a[k] = stage[k * 128 + i];
            const uint32_t acol = tlane + kAlphaCol + (uint32_t)((2 * g + b) * 64 + (jw0 >> 1));
            tmem_st_x8(acol, *(const uint32_t(*)[8])(a));
            tmem_st_x8(acol + 8, *(const uint32_t(*)[8])(a + 8));
            tmem_st_x8(acol + 16, *(const uint32_t(*)[8])(a + 16));
            tmem_st_wait();
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&req[2 * g + b]);
          // ---- P3 of the previous head overlaps this head's gather ----
          if (t >= 1) finish_head(t - 1);
        }
        finish_head(3);
        ok = epilogue_all(ok);
        if (!ok) break;
        if (!last) {
          fence_proxy_async_smem();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(x_ready);
        } else {
          // ---------------- heads (fp32) ----------------
          float* zbuf = (float*)(smem + kSmZ);
          float* logit = (float*)(smem + kSmLogit);
          const int tid = threadIdx.x;  // 0..255
          if (tid < kGPT * 64) {
            const int pg = tid / 64, u = tid % 64;
            float acc = __ldg(p.w + C4Off::b_v1 + u);
            for (int c = 0; c < 256; ++c) acc = fmaf(pooled[pg * 256 + c], __ldg(p.w + C4Off::W_v1 + c * 64 + u), acc);
            zbuf[pg * 64 + u] = fmaxf(acc, 0.f);
          } else if (tid < kGPT * 64 + kGPT * 7) {
            const int k = tid - kGPT * 64, pg = k / 7, c = k % 7;
            float acc = __ldg(p.w + C4Off::b_pi);
            for (int f = 0; f < 256; ++f) acc = fmaf(pcol[(pg * 7 + c) * 256 + f], __ldg(p.w + C4Off::w_pi + f), acc);
            logit[pg * 8 + c] = acc;
          }
          named_bar_sync(1, kEpiWarps * 32);
          if (warp < kGPT) {
            const int pg = warp, pos = tile * kGPT + pg;
            float vv = zbuf[pg * 64 + lane] * __ldg(p.w + C4Off::w_v2 + lane) +
                       zbuf[pg * 64 + 32 + lane] * __ldg(p.w + C4Off::w_v2 + 32 + lane);
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) vv += __shfl_xor_sync(0xffffffffu, vv, o);
            const float lg = lane < 7 ? logit[pg * 8 + lane] : -INFINITY;
            float mx = lg;
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float ex = lane < 7 ? expf(lg - mx) : 0.f;
            float z = ex;
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
            if (pos < p.n) {
              if (lane < 7) p.pi[(size_t)pos * 7 + lane] = ex / z;
              if (lane == 0) p.v[pos] = tanhf(vv + __ldg(p.w + C4Off::b_v2));
            }
          }
          named_bar_sync(1, kEpiWarps * 32);  // head scratch (X tile) free for the next encode
        }
      }
    }
  }

  // ---------------- teardown ----------------
  tc_fence_before();
  __syncthreads();
  if (*abort_flag && threadIdx.x == 0) atomicExch(p.err, 1);
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---- weight packing: W_l^T into swizzled 32 KB chunks [256 features][64 K] ----
template <typename OpT>
__global__ void pack_c4_kernel(const float* __restrict__ w, uint8_t* __restrict__ out) {
  const int chunk = blockIdx.x;  // 0 .. kChunksPerTile-1
  const int layer = chunk == 0 ? 0 : 1 + (chunk - 1) / 4;
  const int c = chunk == 0 ? 0 : (chunk - 1) % 4;
  const int fin = layer == 0 ? 4 : 256;
  const int w_off = layer == 0 ? 0 : C4Off::kLayer0 + (layer - 1) * C4Off::kLayerN;
  const float* W = w + w_off;
  uint8_t* dst = out + (size_t)chunk * kWChunk;
  for (int t = threadIdx.x; t < 256 * 64; t += blockDim.x) {
    const int f = t / 64, kk = t % 64;  // feature row, K within chunk
    const int k = c * 64 + kk;
    const float x = k < fin ? W[(size_t)k * kHidden + f] : 0.f;
    *(uint16_t*)(dst + (f >> 7) * 16384 + sw128_offset(f & 127, kk)) = OpType<OpT>::bits(x);
  }
}

}  // namespace

size_t gat_tc_packed_bytes(int game) { return game == kConnect4 ? (size_t)kChunksPerTile * kWChunk : 0; }

cudaError_t launch_gat_tc_pack(int game, int fp16, const float* d_weights, void* d_packed, cudaStream_t stream) {
  if (game != kConnect4) return cudaErrorNotSupported;
  if (fp16) pack_c4_kernel<__half><<<kChunksPerTile, 256, 0, stream>>>(d_weights, (uint8_t*)d_packed);
  else pack_c4_kernel<__nv_bfloat16><<<kChunksPerTile, 256, 0, stream>>>(d_weights, (uint8_t*)d_packed);
  return cudaGetLastError();
}

cudaError_t launch_gat_tc(int game, int fp16, const void* d_packed, const float* d_weights, const int8_t* d_boards,
                          const int8_t* d_side, int n, float* d_pi, float* d_v, int* d_err, cudaStream_t stream) {
  if (game != kConnect4) return cudaErrorNotSupported;
  if (n <= 0) return cudaSuccess;
  TcParams p;
  p.packed = (const uint8_t*)d_packed;
  p.w = d_weights;
  p.boards = d_boards;
  p.side = d_side;
  p.pi = d_pi;
  p.v = d_v;
  p.err = d_err;
  p.n = n;
  p.num_tiles = (n + kGPT - 1) / kGPT;
  auto kern = fp16 ? gat_tc_c4_kernel<__half> : gat_tc_c4_kernel<__nv_bfloat16>;
  // Per-device persistent grid (one CTA per SM: the CTA owns all 512 tensor
  // memory columns), computed once.
  static int cached_grid[64][2];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  int& full_grid = cached_grid[dev][fp16 ? 1 : 0];
  if (full_grid == 0) {
    int sms = 0;
    if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    full_grid = sms;
  }
  int grid = full_grid < p.num_tiles ? full_grid : p.num_tiles;
  kern<<<grid, kThreads, kSmemBytes, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace gz
