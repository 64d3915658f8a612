// Tensor-core (tcgen05) GAT forward for Connect4: all six layers and both
// heads in one persistent launch, one CTA per SM.
//
// A tile is 128 node rows = 3 positions x 42 nodes (+2 padding rows).  Per
// layer:
//   1. projection   Wh[128 x 256] = X[128 x K] . W[K x 256]       (tcgen05.mma,
//      bf16/fp16 operands from shared memory, fp32 accumulator in tensor
//      memory: lane = node, column = feature), and beside it the attention
//      scores S[128 x 32] = X . (W a): the per-head dot products
//      s_i = a_self . Wh_i^h and t_i = a_nbr . Wh_i^h come out of the same
//      MMA, because a . (x W) = x . (W a).  W a is folded into the packed
//      weights as a bf16 high part and a bf16 remainder (two columns each),
//      so the scores keep fp32-level accuracy in the weights.
//   2. per head h (8 heads, two groups of four run by two warpgroups):
//      softmax  e_ij = exp(LeakyReLU_0.2(s_i + t_j) - max_j), z_i = sum_j e_ij
//               over the 8-neighbourhood + self of node i (the Connect4 board
//               graph); e (fp16, unnormalised) goes into tensor memory, each
//               position's rows relative to a 48-node window that holds the
//               position (neighbours never cross positions)
//      gather   out^h = e^h . Wh^h   as a second tcgen05.mma per position
//               (three K = 16 steps over the window, other lanes disabled):
//               e^h is the A operand in tensor memory, Wh^h (fp16) the B
//               operand in shared memory; the result overwrites the head's
//               accumulator columns
//   3. out / z + bias, ELU, stored as the next layer's X tile (128-byte
//      swizzled, K-major; fp16 rounded to nearest, or bf16 stochastically
//      rounded) -- or, after the last layer, summed in fp32 per (position,
//      board column) straight from the registers: the column sums feed the
//      policy head (256->1 per column, softmax over 7), their totals the
//      value head (256->64 ReLU, 64->1 tanh).
// The next layer's projection does not wait for the head loop: heads c and
// c + 4 write K chunk c of the next X tile, and each chunk's MMAs are issued
// as soon as it exists, into a third accumulator block (tensor memory holds
// three 128-column blocks that rotate from layer to layer).  Between two head
// loops remain the last chunk's score MMAs, which go first, and the
// projection halves of the last two chunks: chunk 2's halves are held back
// until chunk 3's scores are issued, so that the tensor pipe (in order)
// reaches the scores the next head loop starts on without a queue ahead.
// Weights are pre-packed on the device into 36 KB chunks (256 projection rows
// + 32 score rows, 64 K each, swizzled) and streamed into a two-slot
// shared-memory ring by one producer thread with 1-D bulk async copies (TMA
// engine).  Three threads issue MMAs: one the projections, one each group's
// gathers.  Every wait is bounded
// (%globaltimer); on a timeout the CTA drains its copies and MMAs, frees
// tensor memory and reports through the error word.
//
// Reference: networks/gat/gat.cu:836-870 (forward_gat_layer), 916-948
// (compute_output), 995-1038 (softmax, tanh); the math is the standard GAT
// the reference's kernels never completed.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "gz_games.h"
#include "gz_internal.h"
#include "gz_round.h"
#include "gz_sm100.h"

namespace gz {
namespace {

using namespace sm100;

constexpr int kN = 42;              // Connect4 nodes
constexpr int kGPT = 3;             // positions per tile
constexpr int kRows = 128;          // MMA M (node rows per tile)
constexpr int kLayers = 6;
constexpr int kEpiWarps = 8;        // two warpgroups: heads 0-3 and 4-7
constexpr int kThreads = (kEpiWarps + 4) * 32;
constexpr int kProducerWarp = kEpiWarps;
constexpr int kMmaWarp = kEpiWarps + 1;     // group 0's gathers; allocates tensor memory
constexpr int kGatherWarp = kEpiWarps + 2;  // group 1's gathers
constexpr int kProjWarp = kEpiWarps + 3;    // projection and score MMAs
constexpr int kWRows = 256 + 32;    // projection rows + score rows (16 high parts, 16 remainders)
constexpr int kWChunk = kWRows * 128;  // 64 K x 2 B per row
constexpr int kWScoreOff = 256 * 128;  // byte offset of the score rows in a chunk
constexpr int kWSlots = 2;
constexpr int kChunksPerTile = 1 + (kLayers - 1) * 4;
constexpr uint32_t kTmemCols = 512;
// Tensor memory: three 128-column accumulator blocks, the e buffers and the
// score accumulator.  Layer l's projection Wh occupies two blocks: the first
// half (columns of heads 0, 4, 1, 5 in that order: the heads the two groups
// finish first) in block first_block(l), the second half (heads 2, 6, 3, 7)
// in block second_block(l).  Layer l+1's first half accumulates in the third
// block from the moment the first K chunk of X(l+1) exists; its second half
// reuses layer l's first-half block once both groups have finished heads 0
// and 1 (4 and 5), so the next projection runs under the current head loop.
// The blocks rotate with period 3 (six layers per tile: every tile starts
// in the same place).
constexpr uint32_t kECol = 384;      // e buffers: 384 + (2 * group + buffer) * 24
constexpr uint32_t kScoreCol = 480;  // scores: 16 high parts + 16 remainders
__host__ __device__ constexpr int first_block(int l) { return (3 - l % 3) % 3; }
__host__ __device__ constexpr int second_block(int l) { return (4 - l % 3) % 3; }
// head 4g + t of layer l: block by t / 2, slot 2 (t % 2) + g inside it
__host__ __device__ constexpr uint32_t head_col(int l, int g, int t) {
  return (uint32_t)(128 * (t < 2 ? first_block(l) : second_block(l)) + 32 * (2 * (t & 1) + g));
}
static_assert(first_block(kLayers) == first_block(0) && second_block(kLayers) == second_block(0), "rotation period");
constexpr uint64_t kWaitLimitNs = 4000000000ull;  // 4 s per wait
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// Shared memory map (bytes).
constexpr int kStageStride = 112;                       // bytes per staging row (24 used words + pad)
constexpr int kSmX = 0;                                 // X tile: 4 x 16 KB (K-major, 128 rows)
constexpr int kSmW = kSmX + 4 * 16384;                  // weight ring
constexpr int kSmB2 = kSmW + kWSlots * kWChunk;         // Wh^h operand: [group][buffer] 8 KB each
constexpr int kSmStage = kSmB2 + 4 * 8192;              // e staging: [group][128 rows][kStageStride]
constexpr int kSmTsc = kSmStage + 2 * 128 * kStageStride;  // t scores: [group][129][4 heads] floats
constexpr int kSmVec = kSmTsc + 2 * 129 * 16;           // per layer bias[256]; x2 (layer parity)
constexpr int kVecFloats = 256;
constexpr int kSmBar = kSmVec + 2 * kVecFloats * 4;
// full, empty, sc_full, acc_a, acc_b, x_ready[4], req[2][2], done2[2][2], drain[3]
constexpr int kNumBars = 2 * kWSlots + 3 + 4 + 4 + 4 + 3;
constexpr int kSmMisc = kSmBar + kNumBars * 8;
// Last layer: each head's per (position, board column) sums of the
// activations, fp32, as two shares [2][3 positions x 7 columns][32 features]
// (column_partials).  Heads 0, 4, 1, 5 (t = 0, 1) keep them here, heads 2, 6,
// 3, 7 in X chunks 2-3 (read by the projection until its second half is done).
constexpr int kShareBytes = 2 * kGPT * 7 * 32 * 4;  // one head
constexpr int kSmCol = (kSmMisc + 16 + 15) & ~15;
constexpr int kSmemBytes = kSmCol + 4 * kShareBytes;
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
static_assert(kSmW % 1024 == 0 && kWChunk % 1024 == 0, "swizzled tiles need 1024-byte alignment");
// Last-layer head scratch: node means and policy partial sums in the t-score
// region (free once a layer's head loop has its scores), value-head partial
// sums in the X tile once the pooling has read it.
constexpr int kSmMean = kSmTsc;                          // [3][256] floats
constexpr int kSmLgW = kSmMean + kGPT * 256 * 4;         // [8 warps][3 x 7] floats
static_assert(kSmLgW + kEpiWarps * kGPT * 7 * 4 <= kSmVec, "head sums fit in the t-score region");
constexpr int kXZPart = 3 * 16384;                       // X tile offset of [8 warps][3][64] floats
static_assert(kXZPart + kEpiWarps * kGPT * 64 * 4 <= 4 * 16384, "value partials fit in the X tile");
// Last layer: each epilogue warp transposes a head's 32 x 32 activations
// through 4 KB of the X tile (K chunks 0-1, no longer read once the layer's
// first-half projection is complete).
constexpr int kXScratch = 4096;
static_assert(kEpiWarps * kXScratch <= 2 * 16384, "transpose scratch fits in X chunks 0-1");
static_assert(2 * 16384 + 4 * kShareBytes <= 4 * 16384, "column-sum shares of heads t = 2, 3 fit in X chunks 2-3");

// Offsets (floats) into the fp32 weight blob for Connect4 (gat_layout order).
struct C4Off {
  static constexpr int kLayer0 = 4 * 256 + 256 + 512;
  static constexpr int kLayerN = 256 * 256 + 256 + 512;
  __host__ __device__ static constexpr int W(int l) { return l == 0 ? 0 : kLayer0 + (l - 1) * kLayerN; }
  __host__ __device__ static constexpr int b(int l) { return W(l) + (l == 0 ? 4 : 256) * 256; }
  __host__ __device__ static constexpr int a(int l) { return b(l) + 256; }
  static constexpr int kHeads = kLayer0 + (kLayers - 1) * kLayerN;
  static constexpr int w_pi = kHeads, b_pi = w_pi + 256, W_v1 = b_pi + 1, b_v1 = W_v1 + 256 * 64;
  static constexpr int w_v2 = b_v1 + 64, b_v2 = w_v2 + 64;
};

template <typename T> struct OpType;
template <> struct OpType<__nv_bfloat16> {
  static constexpr uint32_t fmt = 1;
  static __device__ __forceinline__ uint16_t bits(float x) { return __bfloat16_as_ushort(__float2bfloat16_rn(x)); }
  static __device__ __forceinline__ float round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  // stochastic rounding: the low element rounds up when rbits[15:0] plus its
  // discarded 16 bits carry, the high element likewise with rbits[31:16]
  static __device__ __forceinline__ uint32_t pack_sr(float lo, float hi, uint32_t rbits) {
    uint32_t d;
    asm("cvt.rs.satfinite.bf16x2.f32 %0, %1, %2, %3;" : "=r"(d) : "f"(hi), "f"(lo), "r"(rbits));
    return d;
  }
};
template <> struct OpType<__half> {
  static constexpr uint32_t fmt = 0;
  static __device__ __forceinline__ uint16_t bits(float x) { return __half_as_ushort(__float2half_rn(x)); }
  static __device__ __forceinline__ float round(float x) { return __half2float(__float2half_rn(x)); }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  static __device__ __forceinline__ uint32_t pack_sr(float lo, float hi, uint32_t rbits) {
    uint32_t d;
    asm("cvt.rs.satfinite.f16x2.f32 %0, %1, %2, %3;" : "=r"(d) : "f"(hi), "f"(lo), "r"(rbits));
    return d;
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

// Random bits for rounding the activations of node `li` (index inside its
// position, so a position rounds the same way in any batch slot), layer l,
// head h.  Identical nodes of one position then round independently, and
// their rounding errors average out in the neighbour gather and the pooling
// instead of adding up (round-to-nearest gives every node of a uniform board
// the same error).
__device__ __forceinline__ uint32_t round_seed(int li, int l, int h) {
  uint32_t x = (uint32_t)li * 0x9E3779B1u + (uint32_t)(l * 8 + h + 1) * 0x85EBCA77u;
  x ^= x >> 15;
  x *= 0x2C1B3C6Du;
  x ^= x >> 12;
  return x;
}
// per feature pair m of a head: seed ^ kPairMix[m] (odd Weyl steps)
__host__ __device__ constexpr uint32_t pair_mix(int m) { return (uint32_t)(m + 1) * 0x9E3779B9u ^ 0x7F4A7C15u; }

__device__ __forceinline__ float comp(const float4& v, int k) {
  return k == 0 ? v.x : k == 1 ? v.y : k == 2 ? v.z : v.w;
}

// Activations are carried multiplied by log2(e) from the first ELU on (the
// next projection, its attention scores and the softmax then work in base 2
// at no cost; the pooled heads multiply by ln 2 once).  For u = y log2(e)
// this returns ELU(y) log2(e) = max((2^(-|u|) - 1) log2(e), u): u for u > 0,
// (e^y - 1) log2(e) otherwise (e^y - 1 >= y everywhere), with no select.
__device__ __forceinline__ float2 elu2_log2e(float2 u) {
  const float2 em = make_float2(ex2_approx(-fabsf(u.x)), ex2_approx(-fabsf(u.y)));
  const float2 m = __ffma2_rn(em, make_float2(kLog2e, kLog2e), make_float2(-kLog2e, -kLog2e));
  return make_float2(fmaxf(m.x, u.x), fmaxf(m.y, u.y));
}

// Last layer, per head: lane d of the epilogue warp with lane quarter QD
// reads feature d of the warp's 32 node rows from the warp's transpose
// scratch (row n: 32 floats, 16-byte units XOR-swizzled by n % 8, so that the
// row writes and the column reads are free of bank conflicts) and sums them
// per (position, board column) in row order.  Every column of position p has
// rows in exactly two warps, lane quarters p and p + 1; the sums go to
// part[share][p * 7 + c][d] with share 0 the lower warp's (QD = p) and share 1
// the upper warp's (QD = p + 1).
// Column-sum shares of head 4g + t (bytes from the shared-memory base).
__host__ __device__ constexpr int share_offset(int g, int t) {
  return (t < 2 ? kSmCol + t * 2 * kShareBytes : kSmX + 2 * 16384 + (t - 2) * 2 * kShareBytes) + g * kShareBytes;
}

template <int QD>
__device__ __forceinline__ void column_partials(const uint8_t* scr, int d, float* part) {
  float v[32];
#pragma unroll
  for (int n = 0; n < 32; ++n) v[n] = *(const float*)(scr + n * 128 + (((d >> 2) ^ (n & 7)) << 4) + (d & 3) * 4);
#pragma unroll
  for (int pc = 0; pc < kGPT * 7; ++pc) {
    const int pos = pc / 7;
    if (pos != QD && pos != QD - 1) continue;
    float sum = 0.f;
    bool any = false;
#pragma unroll
    for (int n = 0; n < 32; ++n) {
      const int i = 32 * QD + n;
      if (i < kGPT * kN && (i / kN) * 7 + (i % kN) % 7 == pc) {
        sum = any ? sum + v[n] : v[n];
        any = true;
      }
    }
    part[((QD - pos) * kGPT * 7 + pc) * 32 + d] = sum;
  }
}

// The e rows of a tile's position p live in tensor memory relative to the
// 48-node window that starts at node window_start(p) (a multiple of 8, so on
// a core-matrix row of Wh^h) and holds the position's 42 nodes: neighbours
// never cross positions.  The padding rows 126, 127 go with position 2.
__host__ __device__ constexpr int window_start(int p) { return p == 0 ? 0 : p == 1 ? 40 : 80; }
__host__ __device__ constexpr int row_position(int i) { return i < kN ? 0 : i < 2 * kN ? 1 : 2; }
// disable-output-lane mask word w of position p: bit set = lane not p's
__host__ __device__ constexpr uint32_t position_mask(int p, int w) {
  uint32_t m = 0;
  for (int b = 0; b < 32; ++b) m |= (row_position(32 * w + b) != p ? 1u : 0u) << b;
  return m;
}

// The gather of one head: wait for its request (e rows and Wh^h staged),
// then per position p three K = 16 steps over the position's window, with
// the other positions' output lanes disabled.  A is the e buffer (row i
// holds e[i][window_start(p) + k] in half-column k), B is Wh^h (fp16,
// N-contiguous) from the window's first node.  Commits to done2.  Returns
// false after an abort or a timed-out wait.
__device__ __forceinline__ bool gather_head(int l, int g, int t, uint32_t tmem, uint64_t b2desc0, uint64_t* req,
                                            uint64_t* done2, uint32_t (&rph)[2], volatile int* abort_flag) {
  constexpr uint32_t idesc2 = idesc_f16(0 /* fp16 */, 128, 32, 1 /* B N-contiguous */);
  const int b = t & 1, ab = 2 * g + b;
  if (!mbar_wait(&req[ab], rph[b] & 1, abort_flag, kWaitLimitNs)) return false;
  ++rph[b];
  tc_fence_after();
  const uint32_t d = tmem + head_col(l, g, t);
  const uint32_t a_col = tmem + kECol + (uint32_t)(ab * 24);
  const uint64_t bd = b2desc0 + (uint64_t)(ab * (8192 >> 4));
#pragma unroll
  for (int p = 0; p < kGPT; ++p) {
    constexpr uint32_t kMasks[kGPT][4] = {
        {position_mask(0, 0), position_mask(0, 1), position_mask(0, 2), position_mask(0, 3)},
        {position_mask(1, 0), position_mask(1, 1), position_mask(1, 2), position_mask(1, 3)},
        {position_mask(2, 0), position_mask(2, 1), position_mask(2, 2), position_mask(2, 3)}};
    const uint64_t bp = bd + (uint64_t)((window_start(p) / 8) * (512 >> 4));
#pragma unroll
    for (int j = 0; j < 3; ++j) mma_f16_ts_masked(d, a_col + 8 * j, bp + j * (1024 >> 4), idesc2, j != 0, kMasks[p]);
  }
  mma_commit(&done2[ab]);
  return true;
}

struct TcParams {
  const uint8_t* packed;  // kChunksPerTile chunks in consumption order
  const float* w;         // fp32 blob (biases, heads)
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
  // a layer's projection complete: scores (sc_full), first-half block
  // (acc_a), second-half block (acc_b), committed in that order
  uint64_t* sc_full = bars + 2 * kWSlots;
  uint64_t* acc_a = sc_full + 1;
  uint64_t* acc_b = sc_full + 2;
  // x_ready[c]: K chunk c of the next X tile written (both groups' head c,
  // c + 4; chunk 0 also marks a tile's encoded input)
  uint64_t* x_ready = sc_full + 3;  // [4 chunks]
  // req / done2 per (group, buffer): a head's gather request and its
  // completion.  One barrier per buffer keeps every producer at most one
  // phase ahead of its consumer.
  uint64_t* req = sc_full + 7;      // [2 groups][2 buffers]
  uint64_t* done2 = sc_full + 11;   // [2 groups][2 buffers]
  uint64_t* drain = sc_full + 15;   // [issuing thread: gathers 0, gathers 1, projection]
  uint32_t* tmem_slot = (uint32_t*)(smem + kSmMisc);
  volatile int* abort_flag = (volatile int*)(smem + kSmMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // zero the e staging (its zero pattern is static), fill the t-score rows
  // of the "no neighbour" node (index 128) with -inf, init barriers
  for (int i = threadIdx.x; i < 2 * 128 * kStageStride / 4; i += blockDim.x) ((uint32_t*)(smem + kSmStage))[i] = 0u;
  if (threadIdx.x < 8) ((float*)(smem + kSmTsc))[(threadIdx.x >> 2) * 129 * 4 + 128 * 4 + (threadIdx.x & 3)] = -INFINITY;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kWSlots; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(sc_full, 1);
    mbar_init(acc_a, 1);
    mbar_init(acc_b, 1);
    for (int i = 0; i < 4; ++i) {
      mbar_init(&x_ready[i], kEpiWarps);
      mbar_init(&req[i], 4);
      mbar_init(&done2[i], 1);
    }
    for (int i = 0; i < 3; ++i) mbar_init(&drain[i], 1);
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
  } else if (warp == kMmaWarp || warp == kGatherWarp) {
    // ---------------- gathers: one issuing thread per group ----------------
    // A head's gather latency is bound by its thread's issue rate, so the
    // two groups' chains run side by side.
    if (lane == 0) {
      const int g = warp - kMmaWarp;
      const uint64_t b2desc0 = noswizzle_desc(smem_u32(smem + kSmB2), 512, 128);
      uint32_t rph[2] = {0, 0};
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x)
        for (int l = 0; l < kLayers && ok; ++l)
          for (int t = 0; t < 4 && ok; ++t) ok = gather_head(l, g, t, tmem, b2desc0, req, done2, rph, abort_flag);
      mma_commit(&drain[g]);
      mbar_wait(&drain[g], 0, abort_flag, kWaitLimitNs);
    }
    __syncwarp();
  } else if (warp == kProjWarp) {
    // ---------------- projection and score MMAs ----------------
    // Layer l + 1's projection is issued chunk by chunk under layer l's head
    // loop, as the K chunks of X(l + 1) appear.  Descriptors are built once
    // and advanced by adding (byte offset >> 4) to the start-address field
    // (no carry out of the 14-bit field: shared addresses stay below 2^18).
    if (lane == 0) {
      constexpr uint32_t idescH = idesc_f16(OpType<OpT>::fmt, 128, 128);
      constexpr uint32_t idesc_s = idesc_f16(OpType<OpT>::fmt, 128, 32);
      const uint64_t xdesc = sw128_desc(smem_u32(sX));
      const uint64_t wdesc0 = sw128_desc(smem_u32(sW));
      uint32_t q = 0, xph[4] = {0, 0, 0, 0};
      bool ok = true;
      auto wait_x = [&](int c) {
        ok = ok && mbar_wait(&x_ready[c], xph[c] & 1, abort_flag, kWaitLimitNs);
        ++xph[c];
        tc_fence_after();
      };
      auto wait_w = [&](uint32_t k) {  // weight chunk k of the stream landed
        ok = ok && mbar_wait(&full[k % kWSlots], (k / kWSlots) & 1, abort_flag, kWaitLimitNs);
        tc_fence_after();
      };
      // K = 16 step kk of X chunk c against weight chunk k: N = 128 into
      // `dcol` from weight rows 128 * half .., or the 32 score columns
      auto proj = [&](uint32_t dcol, int half, int c, uint32_t k, int kk, bool first) {
        const uint64_t xd = xdesc + (uint64_t)(c * (16384 >> 4) + kk * 2);
        const uint64_t wd = wdesc0 + (uint64_t)((k % kWSlots) * (kWChunk >> 4) + kk * 2);
        mma_f16_ss(tmem + dcol, xd, wd + (uint64_t)(half * (16384 >> 4)), idescH, !first);
      };
      auto score = [&](int c, uint32_t k, int kk, bool first) {
        const uint64_t xd = xdesc + (uint64_t)(c * (16384 >> 4) + kk * 2);
        const uint64_t wd = wdesc0 + (uint64_t)((k % kWSlots) * (kWChunk >> 4) + (kWScoreOff >> 4) + kk * 2);
        mma_f16_ss(tmem + kScoreCol, xd, wd, idesc_s, !first);
      };
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        // layer 0: the encoded features (K = 4, one K = 16 step)
        wait_x(0);
        wait_w(q);
        if (!ok) break;
        // the second half goes first: acc_a then covers both halves, and both
        // have read X chunk 0 before head 0's result overwrites it
        score(0, q, 0, true);
        mma_commit(sc_full);
        proj(128 * second_block(0), 1, 0, q, 0, true);
        mma_commit(acc_b);
        proj(128 * first_block(0), 0, 0, q, 0, true);
        mma_commit(acc_a);
        mma_commit(&empty[q % kWSlots]);
        ++q;
        for (int l = 1; l < kLayers && ok; ++l) {
          // layer l from X(l), weight chunks q .. q + 3
          const uint32_t fa = 128 * first_block(l), fb = 128 * second_block(l);
          // chunk 0: first half + scores (the third block is free)
          wait_x(0);
          wait_w(q);
          if (!ok) break;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            proj(fa, 0, 0, q, kk, kk == 0);
            score(0, q, kk, kk == 0);
          }
          // chunk 1: first half + scores; the second half of chunks 0 and 1
          // (layer l-1's first-half block is free: heads 0, 1, 4, 5 done)
          wait_x(1);
          wait_w(q + 1);
          if (!ok) break;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            proj(fa, 0, 1, q + 1, kk, false);
            score(1, q + 1, kk, false);
          }
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) proj(fb, 1, 0, q, kk, kk == 0);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) proj(fb, 1, 1, q + 1, kk, false);
          mma_commit(&empty[q % kWSlots]);
          mma_commit(&empty[(q + 1) % kWSlots]);
          // chunk 2: scores only; its halves wait until chunk 3's scores are
          // issued, so nothing queues ahead of the scores the epilogue waits on
          wait_x(2);
          wait_w(q + 2);
          if (!ok) break;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) score(2, q + 2, kk, false);
          // chunk 3: scores first (the epilogue starts on them), then the
          // first half of chunks 2 and 3, then the second, each committed on
          // its own barrier
          wait_x(3);
          wait_w(q + 3);
          if (!ok) break;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) score(3, q + 3, kk, false);
          mma_commit(sc_full);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) proj(fa, 0, 2, q + 2, kk, false);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) proj(fa, 0, 3, q + 3, kk, false);
          mma_commit(acc_a);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) proj(fb, 1, 2, q + 2, kk, false);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) proj(fb, 1, 3, q + 3, kk, false);
          mma_commit(acc_b);
          mma_commit(&empty[(q + 2) % kWSlots]);
          mma_commit(&empty[(q + 3) % kWSlots]);
          q += 4;
        }
      }
      mma_commit(&drain[2]);
      mbar_wait(&drain[2], 0, abort_flag, kWaitLimitNs);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue: warpgroup g owns heads 4g..4g+3 ----------------
    const int g = warp >> 2, qd = warp & 3;
    const int i = 32 * qd + lane;  // node row of this thread
    const uint32_t tlane = tmem + ((uint32_t)(32 * qd) << 16);
    const int li = i % kN, rr = li / 7, cc = li % 7;
    const bool real = i < kGPT * kN;
    const int jw0 = window_start(row_position(i));
    uint8_t* srow = smem + kSmStage + (g * 128 + i) * kStageStride;
    const float4* tsc = (const float4*)(smem + kSmTsc) + g * 129;
    // node i's 3x3 stencil: the t-score row of each neighbour (128 = none,
    // whose scores are -inf) and the staging address of its e (half-word
    // j - jw0 of row i; absent neighbours write a pad half-word).  Padding
    // rows attend to themselves only.
    int nidx[9];
    uint32_t saddr[9];
#pragma unroll
    for (int k = 0; k < 9; ++k) {
      const int dr = k / 3 - 1, dc = k % 3 - 1;
      const bool in = real ? ((unsigned)(rr + dr) < 6u && (unsigned)(cc + dc) < 7u) : k == 4;
      nidx[k] = in ? i + 7 * dr + dc : 128;
      saddr[k] = smem_u32(srow) + 2 * (in ? i + 7 * dr + dc - jw0 : 48);
    }
    uint32_t aph = 0, dph[2] = {0, 0};
    bool ok = true;    // collective: changes only through epilogue_all
    bool wok = true;   // this thread's waits inside a layer; folded into the next vote


    // Thread t (of 256) encodes the first 16 features (t odd: the zero
    // upper 8) of row t / 2.  Its board cell and side to move are fetched one
    // tile ahead, during the previous tile's last layer, so the encode does
    // not wait on memory.
    static_assert(kEpiWarps * 32 == 2 * kRows, "one encode item per epilogue thread");
    const int ej = threadIdx.x >> 1, ehalf = threadIdx.x & 1, egj = ej / kN, elj = ej % kN;
    int ecell = 0, eside = 1;
    auto fetch_cell = [&](int tile) {
      const int pos = tile * kGPT + egj;
      if (ehalf == 0 && egj < kGPT && tile < p.num_tiles && pos < p.n) {
        ecell = p.boards[(size_t)pos * 42 + elj];
        eside = p.side[pos];
      }
    };
    // encode a tile's positions into X chunk 0 (features 0..15) and release
    // its layer-0 projection.  The first tile is encoded here, every later
    // one during the previous tile's last layer, before its pooling, so that
    // the layer-0 projection and scores run under the pooling and the heads.
    auto encode = [&](int tile) {
      uint32_t wv[4] = {0, 0, 0, 0};
      if (ehalf == 0 && egj < kGPT && tile * kGPT + egj < p.n) {
        const int8_t cell[1] = {(int8_t)ecell};
        float f[4];
        encode_node(kConnect4, cell, eside, 0, f);
        wv[0] = OpType<OpT>::pack(f[0], f[1]);
        wv[1] = OpType<OpT>::pack(f[2], f[3]);
      }
      *(uint4*)(sX + sw128_offset(ej, ehalf * 8)) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&x_ready[0]);
    };
    fetch_cell(blockIdx.x);
    encode(blockIdx.x);
    for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {

      // One layer.  `last` is a compile-time flag, so the last layer's head
      // code does not share registers with the head loop of the others.
      auto layer = [&](int l, auto last_tag) -> bool {
        constexpr bool last = decltype(last_tag)::value;
        if constexpr (last) fetch_cell(tile + gridDim.x);  // the next tile's cells, used after the head loop
        // per-layer bias into shared memory, by layer parity
        float* vec = (float*)(smem + kSmVec) + (l & 1) * kVecFloats;
        vec[threadIdx.x] = __ldg(p.w + C4Off::b(l) + threadIdx.x) * kLog2e;
        const uint32_t lph = aph++ & 1;  // phase of this layer's sc_full / acc_a / acc_b
        wok = mbar_wait(sc_full, lph, abort_flag, kWaitLimitNs) && wok;
        ok = epilogue_all(wok);  // also publishes vec
        if (!ok) return false;
        tc_fence_after();

        // ---- scores of this group's heads: high part + remainder ----
        float s[4];
        {
          float hi[8], lo[8];
          tmem_ld_x8(tlane + kScoreCol + 8 * g, hi);
          tmem_ld_x8(tlane + kScoreCol + 16 + 8 * g, lo);
          tmem_ld_wait();
#pragma unroll
          for (int t = 0; t < 4; ++t) s[t] = hi[2 * t] + lo[2 * t];
          ((float4*)(smem + kSmTsc))[g * 129 + i] =
              make_float4(hi[1] + lo[1], hi[3] + lo[3], hi[5] + lo[5], hi[7] + lo[7]);
        }
        tc_fence_before();
        named_bar_sync(1, kEpiWarps * 32);  // t scores visible; score columns read by everyone
        tc_fence_after();
        float4 tn[9];
#pragma unroll
        for (int k = 0; k < 9; ++k) tn[k] = tsc[nidx[k]];

        float inv[4] = {0.f, 0.f, 0.f, 0.f};

        // P3: result of head t -> / z, + bias, ELU -> next X (or head pooling)
        auto finish_head = [&](int t) {
          const int h = 4 * g + t, b = t & 1;
          wok = mbar_wait(&done2[2 * g + b], dph[b] & 1, abort_flag, kWaitLimitNs) && wok;
          ++dph[b];
          tc_fence_after();
          float o[32];
          tmem_ld_x32(tlane + head_col(l, g, t), o);
          tmem_ld_wait();
          const float4* bias4 = (const float4*)(vec + 32 * h);
          const float2 iv = make_float2(inv[t], inv[t]);
          float2 y[16];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const float4 bv = bias4[k];
            y[2 * k] = elu2_log2e(__ffma2_rn(make_float2(o[4 * k], o[4 * k + 1]), iv, make_float2(bv.x, bv.y)));
            y[2 * k + 1] = elu2_log2e(__ffma2_rn(make_float2(o[4 * k + 2], o[4 * k + 3]), iv, make_float2(bv.z, bv.w)));
          }
          if constexpr (!last) {
            // the next layer's operand: fp16 rounded to nearest; bf16 (8
            // significant bits) stochastically rounded (see round_seed)
            // K chunk t of the next X tile holds heads t (units 0-3) and
            // t + 4 (units 4-7)
            constexpr bool kSr = std::is_same<OpT, __nv_bfloat16>::value;
            const uint32_t seed = kSr ? round_seed(li, l, h) : 0u;
            uint8_t* xrow = sX + t * 16384 + (i >> 3) * 1024 + (i & 7) * 128;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int unit = (4 * g + u) ^ (i & 7);
              uint32_t q[4];
#pragma unroll
              for (int m = 0; m < 4; ++m)
                q[m] = kSr ? OpType<OpT>::pack_sr(y[4 * u + m].x, y[4 * u + m].y, seed ^ pair_mix(4 * u + m))
                           : OpType<OpT>::pack(y[4 * u + m].x, y[4 * u + m].y);
              *(uint4*)(xrow + unit * 16) = make_uint4(q[0], q[1], q[2], q[3]);
            }
            fence_proxy_async_smem();  // X writes -> the next projection's async proxy
            tc_fence_before();         // this head's tensor-memory reads precede the block's reuse
            __syncwarp();
            if (lane == 0) mbar_arrive(&x_ready[t]);
          } else {
            // last layer: the fp32 activations are summed per (position,
            // board column) in fp32: transposed through the warp's scratch
            // into this warp's share of the head's column sums
            // (column_partials); the pooling adds the two shares of every
            // sum in a fixed order, so the result is deterministic
            uint8_t* scr = sX + warp * kXScratch;
#pragma unroll
            for (int j = 0; j < 8; ++j)
              *(float4*)(scr + lane * 128 + ((j ^ (lane & 7)) << 4)) =
                  make_float4(y[2 * j].x, y[2 * j].y, y[2 * j + 1].x, y[2 * j + 1].y);
            __syncwarp();
            float* part = (float*)(smem + share_offset(g, t));  // [2][21][32] floats
            switch (qd) {
              case 0: column_partials<0>(scr, lane, part); break;
              case 1: column_partials<1>(scr, lane, part); break;
              case 2: column_partials<2>(scr, lane, part); break;
              default: column_partials<3>(scr, lane, part); break;
            }
            __syncwarp();       // the scratch is rewritten by the next head
            tc_fence_before();  // this head's tensor-memory reads precede the next tile's projection
          }
        };

        // The head loop always runs to the end (waits return at once after an
        // abort), so every thread meets every named barrier; the decision to
        // stop is collective, at the next layer's start.
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const int b = t & 1;
          // ---- P1: Wh^h (fp32) -> fp16 copy as the gather's B operand ----
          if (t == 0 || t == 2) {  // the block of heads t, t + 1 is complete
            wok = mbar_wait(t == 0 ? acc_a : acc_b, lph, abort_flag, kWaitLimitNs) && wok;
            tc_fence_after();
          }
          {
            float wh[32];
            tmem_ld_x32(tlane + head_col(l, g, t), wh);
            tmem_ld_wait();
            // N-contiguous without swizzle: node i's 8-feature group ng at
            // ng * 128 + (i / 8) * 512 + (i % 8) * 16
            uint8_t* b2 = smem + kSmB2 + (2 * g + b) * 8192 + (i >> 3) * 512 + (i & 7) * 16;
#pragma unroll
            for (int ng = 0; ng < 4; ++ng)
              *(uint4*)(b2 + ng * 128) =
                  make_uint4(OpType<__half>::pack(wh[8 * ng + 0], wh[8 * ng + 1]), OpType<__half>::pack(wh[8 * ng + 2], wh[8 * ng + 3]),
                             OpType<__half>::pack(wh[8 * ng + 4], wh[8 * ng + 5]), OpType<__half>::pack(wh[8 * ng + 6], wh[8 * ng + 7]));
          }
          // ---- P2: neighbour softmax numerators of node i -> e row (fp16) in tensor memory ----
          {
            float lg[9];
            float mx = -INFINITY;
#pragma unroll
            for (int k = 0; k < 9; ++k) {
              const float x = s[t] + comp(tn[k], t);
              lg[k] = fmaxf(x, kLeakySlope * x);
              mx = fmaxf(mx, lg[k]);
            }
            const float c = -mx;  // scores are in base 2 (see elu2_log2e)
            // z sums the fp16 values the gather multiplies, so the weights
            // e / z form an exact convex combination (a uniform neighbourhood
            // reproduces Wh exactly instead of drifting by the rounding of z)
            float z = 0.f;
#pragma unroll
            for (int k = 0; k < 9; ++k) {
              const __half e = __float2half_rn(ex2_approx(lg[k] + c));
              z += __half2float(e);
              asm volatile("st.shared.b16 [%0], %1;" ::"r"(saddr[k]), "h"(__half_as_ushort(e)) : "memory");
            }
            // layer 0 reads the raw features: its Wh carries no log2(e) yet
            inv[t] = rcp_approx(z) * (l == 0 ? kLog2e : 1.f);
            uint32_t a[24];
#pragma unroll
            for (int k = 0; k < 6; ++k) {
              const uint4 v = *(const uint4*)(srow + 16 * k);
              a[4 * k] = v.x;
              a[4 * k + 1] = v.y;
              a[4 * k + 2] = v.z;
              a[4 * k + 3] = v.w;
            }
            const uint32_t acol = tlane + kECol + (uint32_t)((2 * g + b) * 24);
            tmem_st_x8(acol, *(const uint32_t(*)[8])(a));
            tmem_st_x8(acol + 8, *(const uint32_t(*)[8])(a + 8));
            tmem_st_x8(acol + 16, *(const uint32_t(*)[8])(a + 16));
            tmem_st_wait();
          }
          fence_proxy_async_smem();  // B2 writes -> the MMA's async proxy
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&req[2 * g + b]);
          // ---- P3 of the previous head overlaps this head's gather ----
          if (t >= 1) finish_head(t - 1);
        }
        finish_head(3);
        if constexpr (last) {
          // ---------------- heads (fp32) ----------------
          // One pass over the tile's activations: thread f (0..255) owns
          // feature f and sums it over each position's 42 nodes (value head)
          // and over each column's 6 nodes (policy head).  Scales: rows hold
          // ELU log2(e), so means carry ln 2.
          // the value head's weights for this thread (warp w: features
          // 32 w .. 32 w + 31, lane l: units 2 l, 2 l + 1) and the head
          // constants, loaded now so that their latency overlaps the pooling
          float2 wv1[32];
#pragma unroll
          for (int k = 0; k < 32; ++k) {
            const float* src = p.w + C4Off::W_v1 + (32 * warp + k) * 64 + 2 * lane;  // odd offset: scalar loads
            wv1[k] = make_float2(__ldg(src), __ldg(src + 1));
          }
          float hb[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // b_v1 (2), w_v2 (2), b_pi, b_v2
          if (warp < kGPT) {
            hb[0] = __ldg(p.w + C4Off::b_v1 + lane);
            hb[1] = __ldg(p.w + C4Off::b_v1 + 32 + lane);
            hb[2] = __ldg(p.w + C4Off::w_v2 + lane);
            hb[3] = __ldg(p.w + C4Off::w_v2 + 32 + lane);
            hb[4] = __ldg(p.w + C4Off::b_pi);
            hb[5] = __ldg(p.w + C4Off::b_v2);
          }
          named_bar_sync(1, kEpiWarps * 32);  // every head's column sums complete; transpose scratch free
          if (tile + (int)gridDim.x < p.num_tiles) encode(tile + gridDim.x);
          float* mean = (float*)(smem + kSmMean);  // [3][256] node means
          float* lgw = (float*)(smem + kSmLgW);    // [warp][3 x 7] policy partial sums
          {
            const int f = threadIdx.x, hf = f >> 5;
            const float* cs = (const float*)(smem + share_offset(hf >> 2, hf & 3)) + (f & 31);
            float lp[kGPT * 7];
            const float wpf = __ldg(p.w + C4Off::w_pi + f) * (kLn2 / 6.0f);
#pragma unroll
            for (int pg = 0; pg < kGPT; ++pg) {
              float tot = 0.f;
#pragma unroll
              for (int c = 0; c < 7; ++c) {
                const float x = cs[(pg * 7 + c) * 32] + cs[(kGPT * 7 + pg * 7 + c) * 32];
                tot += x;
                lp[pg * 7 + c] = x * wpf;
              }
              mean[pg * 256 + f] = tot * (kLn2 / kN);
            }
            // the warp's 21 policy partials, summed over its lanes and
            // scattered (lane k holds partial k)
            float v32[32];
#pragma unroll
            for (int k = 0; k < 32; ++k) v32[k] = k < kGPT * 7 ? lp[k < kGPT * 7 ? k : 0] : 0.f;
            const float ps = reduce_scatter32(v32, lane);
            if (lane < kGPT * 7) lgw[warp * (kGPT * 7) + lane] = ps;
          }
          named_bar_sync(1, kEpiWarps * 32);  // means and policy partials visible; X tile read
          // value head, first layer: warp w sums features 32 w .. 32 w + 31,
          // lane l units 2 l, 2 l + 1 (each W_v1 element read once per tile)
          float* zpart = (float*)(sX + kXZPart);  // [warp][3][64]
          {
            float a[kGPT][2] = {};
#pragma unroll
            for (int k = 0; k < 32; ++k) {
              const int f = 32 * warp + k;
              const float2 w2 = wv1[k];
#pragma unroll
              for (int pg = 0; pg < kGPT; ++pg) {
                const float m = mean[pg * 256 + f];
                a[pg][0] = fmaf(m, w2.x, a[pg][0]);
                a[pg][1] = fmaf(m, w2.y, a[pg][1]);
              }
            }
#pragma unroll
            for (int pg = 0; pg < kGPT; ++pg)
              *(float2*)(zpart + (warp * kGPT + pg) * 64 + 2 * lane) = make_float2(a[pg][0], a[pg][1]);
          }
          named_bar_sync(1, kEpiWarps * 32);  // value partials visible
          if (warp < kGPT) {
            const int pg = warp, pos = tile * kGPT + pg;
            float z0 = hb[0], z1 = hb[1];
#pragma unroll
            for (int q = 0; q < kEpiWarps; ++q) {
              z0 += zpart[(q * kGPT + pg) * 64 + lane];
              z1 += zpart[(q * kGPT + pg) * 64 + 32 + lane];
            }
            float vv = fmaxf(z0, 0.f) * hb[2] + fmaxf(z1, 0.f) * hb[3];
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) vv += __shfl_xor_sync(0xffffffffu, vv, o);
            float lg = -INFINITY;
            if (lane < 7) {
              lg = hb[4];
#pragma unroll
              for (int q = 0; q < kEpiWarps; ++q) lg += lgw[q * (kGPT * 7) + pg * 7 + lane];
            }
            float mx = lg;
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float ex = lane < 7 ? expf(lg - mx) : 0.f;
            float z = ex;
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
            if (pos < p.n) {
              if (lane < 7) p.pi[(size_t)pos * 7 + lane] = ex / z;
              if (lane == 0) p.v[pos] = tanhf(vv + hb[5]);
            }
          }
          named_bar_sync(1, kEpiWarps * 32);  // head scratch (t-score region, X chunk 3) read by all before the next tile
          // the node means overwrote group 0's "no neighbour" t-score row: restore it
          if (threadIdx.x < 4) ((float*)(smem + kSmTsc))[128 * 4 + threadIdx.x] = -INFINITY;
        }
        return true;
      };
      for (int l = 0; l < kLayers && ok; ++l) {
        const bool cont = l < kLayers - 1 ? layer(l, std::false_type{}) : layer(l, std::true_type{});
        if (!cont) break;
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

// ---- weight packing: 36 KB chunks [288 rows][64 K], 128-byte swizzled ----
// Rows 0..255: W_l^T in the order the accumulator blocks hold the output
// features: rows 32 s .. 32 s + 31 are head (0, 4, 1, 5, 2, 6, 3, 7)[s].
// Rows 256..287: the attention-score weights W_l a_l^h: row 256 + 2h + v
// holds the bf16/fp16 rounding of sum_f W_l[k][32h + f] a_l[h][v][f]
// (v = 0 self, 1 neighbour; times log2(e) for layer 0, whose input is not
// yet carried in base 2), row 272 + 2h + v the rounding of what is left
// over.  K (layers 1..5): chunk c holds the input features of heads c and
// c + 4 (the layer before writes them as its heads finish).
__host__ __device__ constexpr int packed_row_head(int s) { return 4 * (s & 1) + (s >> 1); }

template <typename OpT>
__global__ void pack_c4_kernel(const float* __restrict__ w, uint8_t* __restrict__ out) {
  const int chunk = blockIdx.x;  // 0 .. kChunksPerTile-1
  const int layer = chunk == 0 ? 0 : 1 + (chunk - 1) / 4;
  const int c = chunk == 0 ? 0 : (chunk - 1) % 4;
  const int fin = layer == 0 ? 4 : 256;
  const float* W = w + C4Off::W(layer);
  const float* A = w + C4Off::a(layer);
  uint8_t* dst = out + (size_t)chunk * kWChunk;
  // input feature of K position kk of this chunk
  auto kin = [&](int kk) { return layer == 0 ? kk : 32 * (4 * (kk >> 5) + c) + (kk & 31); };
  for (int t = threadIdx.x; t < 256 * 64; t += blockDim.x) {
    const int r = t / 64, kk = t % 64;  // packed row, K within chunk
    const int f = 32 * packed_row_head(r >> 5) + (r & 31);
    const int k = kin(kk);
    const size_t i = (size_t)k * kHidden + f;
    const float x = k < fin ? W[i] : 0.f;
    *(uint16_t*)(dst + sw128_offset(r, kk)) = weight_bits_sr<OpT>(x, (uint32_t)(C4Off::W(layer) + i));
  }
  for (int t = threadIdx.x; t < 16 * 64; t += blockDim.x) {
    const int j = t / 64, kk = t % 64;  // score column j = 2h + v
    const int k = kin(kk), h = j >> 1, v = j & 1;
    float acc = 0.f;
    if (k < fin)
      for (int f = 0; f < 32; ++f) acc = fmaf(W[(size_t)k * kHidden + 32 * h + f], A[(2 * h + v) * 32 + f], acc);
    if (layer == 0) acc *= kLog2e;  // layer 0's scores in base 2, like the later layers'
    const float hi = OpType<OpT>::round(acc);
    *(uint16_t*)(dst + sw128_offset(256 + j, kk)) = OpType<OpT>::bits(hi);
    *(uint16_t*)(dst + sw128_offset(272 + j, kk)) = OpType<OpT>::bits(acc - hi);
  }
}

}  // namespace

size_t gat_tc_packed_bytes(int game) {
  return game == kConnect4 ? (size_t)kChunksPerTile * kWChunk : game == kChess ? chess_tc_packed_bytes() : 0;
}

cudaError_t launch_gat_tc_pack(int game, int fp16, const float* d_weights, void* d_packed, cudaStream_t stream) {
  if (game == kChess) return launch_chess_tc_pack(fp16, d_weights, d_packed, stream);
  if (game != kConnect4) return cudaErrorNotSupported;
  if (fp16) pack_c4_kernel<__half><<<kChunksPerTile, 256, 0, stream>>>(d_weights, (uint8_t*)d_packed);
  else pack_c4_kernel<__nv_bfloat16><<<kChunksPerTile, 256, 0, stream>>>(d_weights, (uint8_t*)d_packed);
  return cudaGetLastError();
}

cudaError_t launch_gat_tc(int game, int fp16, const void* d_packed, const float* d_weights, const int8_t* d_boards,
                          const int8_t* d_side, int n, float* d_pi, float* d_v, int* d_err, cudaStream_t stream) {
  if (game == kChess) return launch_chess_tc(fp16, d_packed, d_weights, d_boards, d_side, n, d_pi, d_v, d_err, stream);
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
