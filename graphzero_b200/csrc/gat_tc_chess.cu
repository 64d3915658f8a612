// Tensor-core (tcgen05) GAT forward for chess: all eight layers, the
// 4672-way policy and the value head in one persistent launch, one CTA per
// SM.  Same machinery as the Connect4 kernel (gat_tc.cu); what differs:
//
//   * a tile is 128 node rows = 2 positions x 64 squares;
//   * the graph is the static queen-line + knight + self geometry (up to 36
//     neighbours per square, 1856 edges per position), held as a 0/1
//     adjacency table in shared memory; each row's attention weights span
//     its position's 64 squares, i.e. 32 tensor-memory columns of the e
//     buffer, computed from per-square exponential factors (no exponential
//     per edge; see the layer's score phase) and stored from registers;
//   * layer 0 has 18 input features (K padded to 32);
//   * policy: logits[square][73] = X_8[square] . W_pi + b_pi as one more MMA
//     (N = 80, K = 256) on the last layer's activations, softmax over the
//     position's 4672 logits, staged in shared memory and written with one
//     bulk copy per position;
//   * value: mean-pool over the 64 squares (warp reduce-scatter), then the
//     256 -> 64 ReLU -> 1 tanh head in fp32;
//   * as in the Connect4 kernel, layer l + 1's projection runs under layer
//     l's head loop: K chunk t of X(l + 1) holds heads t and t + 4 and its
//     MMAs are issued as soon as both groups have finished head t, into three
//     128-column accumulator blocks that rotate from layer to layer (eight
//     layers a tile, so the rotation follows a layer count that runs on
//     across tiles).  Each group has one e buffer (32 columns: a row's 64
//     squares); a head's e is stored once the group's previous gather has
//     read the buffer.  The gathers run per position (K = 64, the other
//     position's lanes disabled).
//
// Reference: networks/gat/gat.cu:836-870 (forward_gat_layer), 916-948
// (compute_output: per-node 256 -> 73 policy for chess), 995-1038
// (softmax, tanh); action index square * 73 + type (games/chess/chess.cu:96-135).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#include <type_traits>

#include "gz_games.h"
#include "gz_internal.h"
#include "gz_round.h"
#include "gz_sm100.h"

namespace gz {
namespace {

using namespace sm100;

constexpr int kN = 64;              // squares
constexpr int kGPT = 2;             // positions per tile
constexpr int kRows = 128;          // MMA M
constexpr int kLayers = 8;
constexpr int kF = 18;              // input features
constexpr int kP = 73;              // policy outputs per square
constexpr int kPN = 80;             // policy MMA N (73 padded to a multiple of 16)
constexpr int kA = kN * kP;         // 4672 actions
constexpr int kEpiWarps = 8;
constexpr int kThreads = (kEpiWarps + 4) * 32;
constexpr int kProducerWarp = kEpiWarps;
constexpr int kMmaWarp = kEpiWarps + 1;     // projection + policy MMAs + group 0's gathers
constexpr int kGatherWarp = kEpiWarps + 2;  // group 1's gathers
constexpr int kProjWarp = kEpiWarps + 3;    // projection, score and policy MMAs
constexpr int kWRows = 256 + 32;            // projection rows + score rows
constexpr int kWChunk = kWRows * 128;       // 36 KB: 288 rows x 64 K x 2 B
constexpr int kWScoreOff = 256 * 128;
constexpr int kPolChunk = kPN * 128;        // 10 KB: 80 rows x 64 K x 2 B
constexpr int kWSlots = 2;
constexpr int kLayerChunks = 1 + (kLayers - 1) * 4;     // 29
constexpr int kChunksPerTile = kLayerChunks + 4;        // + 4 policy chunks
constexpr uint32_t kTmemCols = 512;
// Tensor memory: three 128-column projection blocks (0-383), the two
// groups' e buffers (384 + 32 g) and the scores (448).  Layer L (counted
// across tiles) keeps heads 0, 4, 1, 5 (t = 0, 1 of both groups) in block
// first_block(L) and heads 2, 6, 3, 7 in second_block(L); layer L + 1's
// first half goes to the third block while layer L's heads run, its second
// half to layer L's first-half block once heads t = 0, 1 are finished.  The
// policy accumulator (80 columns) takes the block after the last layer's.
constexpr uint32_t kECol = 384;
constexpr uint32_t kScoreCol = 448;  // 16 high parts + 16 remainders
__host__ __device__ constexpr int first_block(int L) { return (3 - L % 3) % 3; }
__host__ __device__ constexpr int second_block(int L) { return (4 - L % 3) % 3; }
// head 4g + t of layer L: block by t / 2, slot 2 (t % 2) + g inside it
__host__ __device__ constexpr uint32_t head_col(int L, int g, int t) {
  return (uint32_t)(128 * (t < 2 ? first_block(L) : second_block(L)) + 32 * (2 * (t & 1) + g));
}
constexpr uint64_t kWaitLimitNs = 4000000000ull;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
// Rows whose neighbour maximum lies more than this many (base-2) score units
// below the maximum of a half board take the direct exponentials: the
// product form's factors would leave the fp32 range.  The environment
// variable GZ_CHESS_FACTOR_GAP overrides it at launch (a negative value
// sends every row through the direct path; both paths compute the same
// numerators).
constexpr float kMaxFactorGap = 64.f;

// Knight move k of 8 as (row, column) steps.
__host__ __device__ constexpr int knight_dr(int k) { return k < 4 ? (k == 0 || k == 3 ? 1 : 2) : (k == 4 || k == 7 ? -1 : -2); }
__host__ __device__ constexpr int knight_dc(int k) { return (k == 0 || k == 7) ? 2 : (k == 1 || k == 6) ? 1 : (k == 2 || k == 5) ? -1 : -2; }

// Shared memory map (bytes).
constexpr int kSmX = 0;                                 // X tile 64 KB; after the policy MMA: pi staging
constexpr int kSmW = kSmX + 4 * 16384;
constexpr int kSmB2 = kSmW + kWSlots * kWChunk;
// board graph adjacency as 0/1 factors: row s, 16-byte unit u (squares
// 4u .. 4u + 3) at unit u ^ (s & 15), so that 8 consecutive squares' reads
// of one unit fall in 8 different bank groups
constexpr int kSmMask = kSmB2 + 4 * 8192;
constexpr int kSmT = kSmMask + 64 * 64 * 4;                  // t scores [group][position][head][64]
constexpr int kSmBD = kSmT + 2 * kGPT * 4 * 64 * 4;          // [group][position][head][B: 64 | D: 64]
constexpr int kSmLines = kSmBD + 2 * kGPT * 4 * 128 * 4;     // diagonal maxima [group][position][head][2][16]
constexpr int kSmCol = kSmLines + 2 * kGPT * 4 * 2 * 16 * 4; // column maxima of a warp's 4 rows [group][quarter][head][8]
constexpr int kSmRef = kSmCol + 2 * 4 * 4 * 8 * 4;          // maxima of a warp's 32 squares [group][quarter][head]
constexpr int kSmVec = kSmRef + 2 * 4 * 4 * 4;
constexpr int kVecFloats = 256;
constexpr int kSmPool = kSmVec + 2 * kVecFloats * 4;    // [2 groups][4 quarters][32] node sums of one head
constexpr int kSmZ = kSmPool + 2 * 4 * 32 * 4;          // [2 groups][2 halves][2 pos][64] value partial sums
constexpr int kSmRed = kSmZ + 2 * 2 * kGPT * 64 * 4;    // [4 quarters][2] policy max / sum exchange
constexpr int kSmBar = (kSmRed + 4 * 2 * 4 + 7) & ~7;
// full, empty, sc_full, acc_a, acc_b, x_ready[4], req[2][2], done2[2][2], drain[3], pol_full
constexpr int kNumBars = 2 * kWSlots + 3 + 4 + 4 + 4 + 3 + 1;
constexpr int kSmMisc = kSmBar + kNumBars * 8;
constexpr int kSmemBytes = kSmMisc + 16;
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
static_assert(kSmW % 1024 == 0 && kWChunk % 1024 == 0, "swizzled tiles need 1024-byte alignment");
static_assert(kGPT * kA * 4 <= kSmW, "policy staging fits in the X tile");

// Offsets (floats) into the fp32 weight blob for chess (gat_layout order).
struct ChOff {
  static constexpr int kLayer0 = kF * 256 + 256 + 512;
  static constexpr int kLayerN = 256 * 256 + 256 + 512;
  __host__ __device__ static constexpr int W(int l) { return l == 0 ? 0 : kLayer0 + (l - 1) * kLayerN; }
  __host__ __device__ static constexpr int b(int l) { return W(l) + (l == 0 ? kF : 256) * 256; }
  __host__ __device__ static constexpr int a(int l) { return b(l) + 256; }
  static constexpr int kHeads = kLayer0 + (kLayers - 1) * kLayerN;
  static constexpr int w_pi = kHeads, b_pi = w_pi + 256 * kP, W_v1 = b_pi + kP, b_v1 = W_v1 + 256 * 64;
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

// Random bits for stochastically rounding node `li` (square, so a position
// rounds the same way in any batch slot), layer l, head h; see gat_tc.cu.
__device__ __forceinline__ uint32_t round_seed(int li, int l, int h) {
  uint32_t x = (uint32_t)li * 0x9E3779B1u + (uint32_t)(l * 8 + h + 1) * 0x85EBCA77u;
  x ^= x >> 15;
  x *= 0x2C1B3C6Du;
  x ^= x >> 12;
  return x;
}
__host__ __device__ constexpr uint32_t pair_mix(int m) { return (uint32_t)(m + 1) * 0x9E3779B9u ^ 0x7F4A7C15u; }

// Activations are carried multiplied by log2(e) from the first ELU on (the
// next projection, its attention scores, the softmax and the policy softmax
// then work in base 2 at no cost; the value head multiplies by ln 2 once).
// For u = y log2(e) this returns ELU(y) log2(e) = max((2^(-|u|) - 1) log2(e), u).
__device__ __forceinline__ float2 elu2_log2e(float2 u) {
  const float2 em = make_float2(ex2_approx(-fabsf(u.x)), ex2_approx(-fabsf(u.y)));
  const float2 m = __ffma2_rn(em, make_float2(kLog2e, kLog2e), make_float2(-kLog2e, -kLog2e));
  return make_float2(fmaxf(m.x, u.x), fmaxf(m.y, u.y));
}

// One group's four gathers of layer L (see gat_tc.cu): wait for head t's
// request, then per position four K = 16 steps over its 64 squares (A: the
// group's e buffer, row i holding its position's e in half-column k; B:
// Wh^h from the position's first node; the other position's lanes
// disabled), commit to done2.
__device__ __forceinline__ bool serve_gathers(int L, int g, uint32_t tmem, uint64_t b2desc0, uint64_t* req,
                                              uint64_t* done2, uint32_t (&rph)[2], volatile int* abort_flag) {
  constexpr uint32_t idesc2 = idesc_f16(0 /* fp16 */, 128, 32, 1 /* B N-contiguous */);
  constexpr uint32_t kMasks[kGPT][4] = {{0u, 0u, ~0u, ~0u}, {~0u, ~0u, 0u, 0u}};  // bit set = lane skipped
  const uint32_t a_col = tmem + kECol + (uint32_t)(32 * g);
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const int b = t & 1, ab = 2 * g + b;
    if (!mbar_wait(&req[ab], rph[b] & 1, abort_flag, kWaitLimitNs)) return false;
    ++rph[b];
    tc_fence_after();
    const uint32_t d = tmem + head_col(L, g, t);
    const uint64_t bd = b2desc0 + (uint64_t)(ab * (8192 >> 4));
#pragma unroll
    for (int pg = 0; pg < kGPT; ++pg) {
      const uint64_t bp = bd + (uint64_t)(pg * 8 * (512 >> 4));  // node 64 pg: 8 groups of 8 nodes, 512 B apart
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        mma_f16_ts_masked(d, a_col + kk * 8, bp + kk * (1024 >> 4), idesc2, kk != 0, kMasks[pg]);
    }
    mma_commit(&done2[ab]);
  }
  return true;
}

// 1-D bulk copy shared -> global (TMA engine), tracked by the issuing
// thread's bulk group.
__device__ __forceinline__ void bulk_s2g(void* dst_gmem, const void* src_smem, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst_gmem), "r"(smem_u32(src_smem)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until the committed bulk copies have finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Waits until the committed bulk copies are complete (writes visible).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

struct TcParams {
  const uint8_t* packed;
  const float* w;
  const int8_t* boards;
  const int8_t* side;
  float* pi;
  float* v;
  int* err;
  int n;
  int num_tiles;
  float max_gap;  // kMaxFactorGap or its override
};

template <typename OpT>
__global__ void __launch_bounds__(kThreads, 1) gat_tc_chess_kernel(TcParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) atomicExch(p.err, 2);
    return;
  }
  uint8_t* sX = smem + kSmX;
  uint8_t* sW = smem + kSmW;
  uint64_t* bars = (uint64_t*)(smem + kSmBar);
  uint64_t* full = bars;
  uint64_t* empty = bars + kWSlots;
  // sc_full: a layer's scores complete; acc_a / acc_b: its first / second
  // projection half; x_ready[c]: K chunk c of the next X written (all eight
  // epilogue warps); req / done2 per (group, B2 buffer): a head's gather
  // request and its completion
  uint64_t* sc_full = bars + 2 * kWSlots;
  uint64_t* acc_a = sc_full + 1;
  uint64_t* acc_b = sc_full + 2;
  uint64_t* x_ready = sc_full + 3;  // [4 chunks]
  uint64_t* req = sc_full + 7;      // [2 groups][2 buffers]
  uint64_t* done2 = sc_full + 11;   // [2 groups][2 buffers]
  uint64_t* drain = sc_full + 15;   // [issuing thread: gathers 0, gathers 1, projection]
  uint64_t* pol_full = sc_full + 18;
  uint32_t* tmem_slot = (uint32_t*)(smem + kSmMisc);
  volatile int* abort_flag = (volatile int*)(smem + kSmMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  for (int k = threadIdx.x; k < 64 * 64; k += blockDim.x) {
    const int s = k >> 6, j = k & 63;
    ((float*)(smem + kSmMask))[s * 64 + (((j >> 2) ^ (s & 15)) << 2) + (j & 3)] =
        graph_adjacent(kChess, 8, 8, s, j) ? 1.f : 0.f;
  }
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
    mbar_init(pol_full, 1);
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
          const uint32_t bytes = c < kLayerChunks ? kWChunk : kPolChunk;
          const size_t off = c < kLayerChunks ? (size_t)c * kWChunk
                                              : (size_t)kLayerChunks * kWChunk + (size_t)(c - kLayerChunks) * kPolChunk;
          ok = mbar_wait(&empty[s], ((q / kWSlots) & 1) ^ 1, abort_flag, kWaitLimitNs);
          if (!ok) break;
          mbar_arrive_expect_tx(&full[s], bytes);
          bulk_g2s(sW + s * kWChunk, p.packed + off, bytes, &full[s]);
        }
      }
      for (uint32_t k = (q > kWSlots ? q - kWSlots : 0); k < q; ++k)
        mbar_wait(&full[k % kWSlots], (k / kWSlots) & 1, abort_flag, kWaitLimitNs);
    }
    __syncwarp();
  } else if (warp == kMmaWarp || warp == kGatherWarp) {
    // ---------------- gathers: one issuing thread per group ----------------
    if (lane == 0) {
      const int g = warp - kMmaWarp;
      const uint64_t b2desc0 = noswizzle_desc(smem_u32(smem + kSmB2), 512, 128);
      uint32_t rph[2] = {0, 0};
      bool ok = true;
      int L = 0;  // layers counted across tiles: the projection blocks rotate with it
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x)
        for (int l = 0; l < kLayers && ok; ++l, ++L) ok = serve_gathers(L, g, tmem, b2desc0, req, done2, rph, abort_flag);
      mma_commit(&drain[g]);
      mbar_wait(&drain[g], 0, abort_flag, kWaitLimitNs);
    }
    __syncwarp();
  } else if (warp == kProjWarp) {
    // ---------------- projection, score and policy MMAs ----------------
    // Layer L + 1's projection is issued chunk by chunk under layer L's head
    // loop, as the K chunks of X(L + 1) appear (the Connect4 kernel's order:
    // gat_tc.cu).  Descriptors are advanced by adding (byte offset >> 4) to
    // the start-address field.
    if (lane == 0) {
      constexpr uint32_t idescH = idesc_f16(OpType<OpT>::fmt, 128, 128);
      constexpr uint32_t idesc_s = idesc_f16(OpType<OpT>::fmt, 128, 32);
      constexpr uint32_t idesc_p = idesc_f16(OpType<OpT>::fmt, 128, kPN);
      const uint64_t xdesc = sw128_desc(smem_u32(sX));
      const uint64_t wdesc0 = sw128_desc(smem_u32(sW));
      uint32_t q = 0, xph[4] = {0, 0, 0, 0};
      bool ok = true;
      int L = 0;
      auto wait_x = [&](int c) {
        ok = ok && mbar_wait(&x_ready[c], xph[c] & 1, abort_flag, kWaitLimitNs);
        ++xph[c];
        tc_fence_after();
      };
      auto wait_w = [&](uint32_t k) {  // weight chunk k of the stream landed
        ok = ok && mbar_wait(&full[k % kWSlots], (k / kWSlots) & 1, abort_flag, kWaitLimitNs);
        tc_fence_after();
      };
      auto xd = [&](int c, int kk) { return xdesc + (uint64_t)(c * (16384 >> 4) + kk * 2); };
      auto wd = [&](uint32_t k, int kk) { return wdesc0 + (uint64_t)((k % kWSlots) * (kWChunk >> 4) + kk * 2); };
      // K = 16 step kk of X chunk c against weight chunk k: N = 128 into
      // `dcol` from weight rows 128 * half .., or the 32 score columns
      auto proj = [&](uint32_t dcol, int half, int c, uint32_t k, int kk, bool first) {
        mma_f16_ss(tmem + dcol, xd(c, kk), wd(k, kk) + (uint64_t)(half * (16384 >> 4)), idescH, !first);
      };
      auto score = [&](int c, uint32_t k, int kk, bool first) {
        mma_f16_ss(tmem + kScoreCol, xd(c, kk), wd(k, kk) + (uint64_t)(kWScoreOff >> 4), idesc_s, !first);
      };
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        // layer 0: the encoded features (18 of K = 32: two K = 16 steps)
        {
          const uint32_t fa = 128 * first_block(L), fb = 128 * second_block(L);
          wait_x(0);
          wait_w(q);
          if (!ok) break;
          // the second half goes first: acc_a then covers both halves, and
          // both have read X chunk 0 before head 0's result overwrites it
          for (int kk = 0; kk < 2; ++kk) score(0, q, kk, kk == 0);
          mma_commit(sc_full);
          for (int kk = 0; kk < 2; ++kk) proj(fb, 1, 0, q, kk, kk == 0);
          mma_commit(acc_b);
          for (int kk = 0; kk < 2; ++kk) proj(fa, 0, 0, q, kk, kk == 0);
          mma_commit(acc_a);
          mma_commit(&empty[q % kWSlots]);
          ++q;
          ++L;
        }
        for (int l = 1; l < kLayers && ok; ++l, ++L) {
          // layer L from X, weight chunks q .. q + 3
          const uint32_t fa = 128 * first_block(L), fb = 128 * second_block(L);
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
          // (layer L - 1's first-half block is free: heads 0, 1, 4, 5 done)
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
          // chunk 3: scores first, then the first half of chunks 2 and 3, then
          // the second, each committed on its own barrier
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
        if (!ok) break;
        // policy: X(8) chunk by chunk, N = 80 into the block after the last
        // layer's (free: its last use was layer L - 2's second half)
        const uint32_t pcol = 128 * first_block(L);
        for (int c = 0; c < 4 && ok; ++c) {
          wait_x(c);
          wait_w(q + c);
          if (!ok) break;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) mma_f16_ss(tmem + pcol, xd(c, kk), wd(q + c, kk), idesc_p, (c | kk) != 0);
          mma_commit(&empty[(q + c) % kWSlots]);
        }
        mma_commit(pol_full);
        q += 4;
      }
      mma_commit(&drain[2]);
      mbar_wait(&drain[2], 0, abort_flag, kWaitLimitNs);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue: warpgroup g owns heads 4g..4g+3 ----------------
    const int g = warp >> 2, qd = warp & 3;
    const int i = 32 * qd + lane;        // node row
    const int pg = i >> 6, sq = i & 63;  // position slot in the tile, square
    const uint32_t tlane = tmem + ((uint32_t)(32 * qd) << 16);
    const int br = sq >> 3, bc = sq & 7;  // board row and column
    // this row's position: t scores, B / D factors and diagonal maxima (head 0)
    float* sT = (float*)(smem + kSmT) + (g * kGPT + pg) * 4 * 64;
    float* sBD = (float*)(smem + kSmBD) + (g * kGPT + pg) * 4 * 128;
    const float* sLn = (const float*)(smem + kSmLines) + (g * kGPT + pg) * 4 * 32;
    float* sCol = (float*)(smem + kSmCol) + g * 4 * 4 * 8;
    float* sRef = (float*)(smem + kSmRef) + g * 4 * 4;
    const float* mrow = (const float*)(smem + kSmMask) + sq * 64;
    // knight moves that stay on the board (bit k)
    uint32_t kvalid = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k)
      kvalid |= ((unsigned)(br + knight_dr(k)) < 8u && (unsigned)(bc + knight_dc(k)) < 8u ? 1u : 0u) << k;
    const int gbar = 3 + g;
    uint32_t aph = 0, pph = 0, dph[2] = {0, 0};
    bool ok = true, wok = true;
    int L = 0;  // layers counted across tiles (projection block rotation)

    for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
      // -- encode the tile's positions into X chunk 0 (K = 0..31: 18 features, zeros) --
      for (int t = threadIdx.x; t < kRows * 4; t += kEpiWarps * 32) {
        const int j = t >> 2, unit = t & 3;
        const int gj = j >> 6, lj = j & 63;
        const int pos = tile * kGPT + gj;
        uint32_t wv[4] = {0, 0, 0, 0};
        if (unit < 3 && pos < p.n) {
          float f[kF];
          encode_node(kChess, p.boards + (size_t)pos * 66, p.side[pos], lj, f);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int k0 = unit * 8 + 2 * e;
            wv[e] = OpType<OpT>::pack(k0 < kF ? f[k0 < kF ? k0 : 0] : 0.f, k0 + 1 < kF ? f[k0 + 1 < kF ? k0 + 1 : 0] : 0.f);
          }
        }
        *(uint4*)(sX + sw128_offset(j, unit * 8)) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();  // the previous tile's policy reads precede this tile's layer-0 MMAs
      __syncwarp();
      if (lane == 0) mbar_arrive(&x_ready[0]);

      const int gt = threadIdx.x & 127, vu = gt & 63, vhalf = gt >> 6;
      float* zacc = (float*)(smem + kSmZ) + (g * 2 + vhalf) * kGPT * 64 + vu;  // [pg * 64]

      auto layer = [&](int l, auto last_tag) -> bool {
        constexpr bool last = decltype(last_tag)::value;
        float* vec = (float*)(smem + kSmVec) + (l & 1) * kVecFloats;
        vec[threadIdx.x] = __ldg(p.w + ChOff::b(l) + threadIdx.x) * kLog2e;
        const uint32_t lph = aph++ & 1;  // phase of this layer's sc_full / acc_a / acc_b
        wok = mbar_wait(sc_full, lph, abort_flag, kWaitLimitNs) && wok;
        ok = epilogue_all(wok);
        if (!ok) return false;
        tc_fence_after();

        // ---- scores: s (this row attending), t (this square as a neighbour) ----
        // e_ij = 2^(LeakyReLU(s_i + t_j) + c_i) over the neighbours j of i,
        // with c_i = -LeakyReLU(s_i + max_j t_j) (LeakyReLU is monotonic).
        // With r_h the maximum of t over half board h (one warp's 32 squares),
        // per square B_j = 2^(t_j - r_h), D_j = 2^(0.2 (t_j - r_h)) and per
        // row A_i = 2^(s_i + r_h + c_i), C_i = 2^(0.2 (s_i + r_h) + c_i):
        // e_ij = max(A_i B_j, C_i D_j) -- two exponentials per square and
        // head, four per row, instead of one per edge.  The neighbours'
        // maximum is that of the square's row, column, diagonal, anti-diagonal
        // (the queen lines of the graph) and knight squares.
        float s[4], cs[4];
        uint32_t fb = 0;  // bit t: this row takes head t's direct exponentials
        {
          float hi[8], lo[8];
          tmem_ld_x8(tlane + kScoreCol + 8 * g, hi);
          tmem_ld_x8(tlane + kScoreCol + 16 + 8 * g, lo);
          tmem_ld_wait();
          float rmax[4], cmax[4];
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            s[t] = hi[2 * t] + lo[2 * t];
            const float tv = hi[2 * t + 1] + lo[2 * t + 1];
            sT[t * 64 + sq] = tv;
            // board row (8 lanes), the column over the warp's 4 rows, the warp
            float m = fmaxf(tv, __shfl_xor_sync(~0u, tv, 1));
            m = fmaxf(m, __shfl_xor_sync(~0u, m, 2));
            m = fmaxf(m, __shfl_xor_sync(~0u, m, 4));
            rmax[t] = m;
            float cm = fmaxf(tv, __shfl_xor_sync(~0u, tv, 8));
            cm = fmaxf(cm, __shfl_xor_sync(~0u, cm, 16));
            cmax[t] = cm;
            float wm = fmaxf(m, __shfl_xor_sync(~0u, m, 8));
            wm = fmaxf(wm, __shfl_xor_sync(~0u, wm, 16));
            if (lane < 8) sCol[(qd * 4 + t) * 8 + lane] = cm;
            if (lane == 0) sRef[qd * 4 + t] = wm;
            const float d = tv - wm;
            sBD[t * 128 + sq] = ex2_approx(d);
            sBD[t * 128 + 64 + sq] = ex2_approx(kLeakySlope * d);
          }
          tc_fence_before();
          named_bar_sync(1, kEpiWarps * 32);  // tables written; score columns read by everyone
          tc_fence_after();
          // the other half board's part of the column, and the knight squares
          float nmax[4];
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            float m = fmaxf(fmaxf(rmax[t], cmax[t]), sCol[((qd ^ 1) * 4 + t) * 8 + bc]);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const int j = (kvalid >> k) & 1u ? sq + 8 * knight_dr(k) + knight_dc(k) : sq;
              m = fmaxf(m, sT[t * 64 + j]);
            }
            nmax[t] = m;
          }
          // diagonal and anti-diagonal maxima of the group's two positions
          // and four heads: 240 lines over the group's 128 threads
          for (int task = threadIdx.x & 127; task < kGPT * 4 * 30; task += 128) {
            const int tp = task / 120, rem = task % 120, t = rem / 30, kind = (rem % 30) / 15, d = rem % 15;
            const float* tt = (const float*)(smem + kSmT) + ((g * kGPT + tp) * 4 + t) * 64;
            float m = -INFINITY;
#pragma unroll
            for (int rr = 0; rr < 8; ++rr) {
              const int cc = kind == 0 ? rr + 7 - d : d - rr;  // r - c = d - 7, or r + c = d
              if ((unsigned)cc < 8u) m = fmaxf(m, tt[rr * 8 + cc]);
            }
            ((float*)(smem + kSmLines))[((g * kGPT + tp) * 4 + t) * 32 + kind * 16 + d] = m;
          }
          named_bar_sync(gbar, 128);
          const int qlo = qd & ~1;
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const float m = fmaxf(nmax[t], fmaxf(sLn[t * 32 + br - bc + 7], sLn[t * 32 + 16 + br + bc]));
            const float x = s[t] + m;
            cs[t] = -fmaxf(x, kLeakySlope * x);
            if (fmaxf(sRef[qlo * 4 + t], sRef[(qlo + 1) * 4 + t]) - m > p.max_gap) fb |= 1u << t;
          }
        }
        float inv[4] = {0.f, 0.f, 0.f, 0.f};

        // head t's gather complete: its result may be read, and the group's
        // e buffer rewritten
        auto wait_gather = [&](int t) {
          const int b = t & 1;
          wok = mbar_wait(&done2[2 * g + b], dph[b] & 1, abort_flag, kWaitLimitNs) && wok;
          ++dph[b];
          tc_fence_after();
        };

        // result of head t (after wait_gather(t)) -> / z, + bias, ELU -> K
        // chunk t of the next X (heads t and t + 4)
        auto finish_head = [&](int t) {
          const int h = 4 * g + t;
          float o[32];
          tmem_ld_x32(tlane + head_col(L, g, t), o);
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
          // next layer's operand (the last layer's feeds the policy MMA):
          // fp16 rounded to nearest, bf16 stochastically rounded (round_seed)
          {
            constexpr bool kSr = std::is_same<OpT, __nv_bfloat16>::value;
            const uint32_t seed = kSr ? round_seed(sq, l, h) : 0u;
            uint8_t* xrow = sX + t * 16384 + (i >> 3) * 1024 + (i & 7) * 128;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int unit = (4 * g + u) ^ (i & 7);
              uint32_t qv[4];
#pragma unroll
              for (int m = 0; m < 4; ++m)
                qv[m] = kSr ? OpType<OpT>::pack_sr(y[4 * u + m].x, y[4 * u + m].y, seed ^ pair_mix(4 * u + m))
                            : OpType<OpT>::pack(y[4 * u + m].x, y[4 * u + m].y);
              *(uint4*)(xrow + unit * 16) = make_uint4(qv[0], qv[1], qv[2], qv[3]);
            }
          }
          fence_proxy_async_smem();  // X writes -> the next projection's (or the policy MMA's) async proxy
          tc_fence_before();         // this head's tensor-memory reads precede the block's reuse
          __syncwarp();
          if (lane == 0) mbar_arrive(&x_ready[t]);
          if constexpr (last) {
            // value head: node sums of this head (fp32), per position
            float v32[32];
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              v32[2 * k] = y[k].x;
              v32[2 * k + 1] = y[k].y;
            }
            const float sum = reduce_scatter32(v32, lane);  // lane d: sum of feature d over this warp's rows
            float* pool = (float*)(smem + kSmPool) + (g * 4 + qd) * 32;
            pool[lane] = sum;
            named_bar_sync(gbar, 128);
            float wv[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) wv[j] = __ldg(p.w + ChOff::W_v1 + (32 * h + 16 * vhalf + j) * 64 + vu);
#pragma unroll
            for (int q2 = 0; q2 < kGPT; ++q2) {
              const float* pa = (const float*)(smem + kSmPool) + (g * 4 + 2 * q2) * 32;
              float acc = t == 0 ? 0.f : zacc[q2 * 64];
#pragma unroll
              for (int j = 0; j < 16; ++j)
                acc = fmaf((pa[16 * vhalf + j] + pa[32 + 16 * vhalf + j]) * (kLn2 / kN), wv[j], acc);
              zacc[q2 * 64] = acc;
            }
            named_bar_sync(gbar, 128);  // pool slots reused by the next head
          }
        };

#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const int b = t & 1;
          {  // P1: Wh^h (fp32) -> fp16 B operand of the gather
            if (t == 0 || t == 2) {  // the block of heads t, t + 1 is complete
              wok = mbar_wait(t == 0 ? acc_a : acc_b, lph, abort_flag, kWaitLimitNs) && wok;
              tc_fence_after();
            }
            float wh[32];
            tmem_ld_x32(tlane + head_col(L, g, t), wh);
            tmem_ld_wait();
            uint8_t* b2 = smem + kSmB2 + (2 * g + b) * 8192 + (i >> 3) * 512 + (i & 7) * 16;
#pragma unroll
            for (int ng = 0; ng < 4; ++ng)
              *(uint4*)(b2 + ng * 128) =
                  make_uint4(OpType<__half>::pack(wh[8 * ng + 0], wh[8 * ng + 1]), OpType<__half>::pack(wh[8 * ng + 2], wh[8 * ng + 3]),
                             OpType<__half>::pack(wh[8 * ng + 4], wh[8 * ng + 5]), OpType<__half>::pack(wh[8 * ng + 6], wh[8 * ng + 7]));
          }
          {  // P2: softmax numerators over the position's 64 squares -> e row (fp16)
            const float st = s[t], ct = cs[t];
            uint32_t e2[32];
            float2 z2 = make_float2(0.f, 0.f);
            // squares 4q .. 4q + 3 -> e row words 2q, 2q + 1; z sums the fp32 values
            auto put = [&](int q, float2 e01, float2 e23) {
              z2 = __fadd2_rn(z2, __fadd2_rn(e01, e23));
              e2[2 * q] = OpType<__half>::pack(e01.x, e01.y);
              e2[2 * q + 1] = OpType<__half>::pack(e23.x, e23.y);
            };
            if (__any_sync(~0u, (fb >> t) & 1u)) {
              // one exponential per square, off-graph squares at -inf
              const float* tt = sT + t * 64;
#pragma unroll
              for (int q = 0; q < 16; ++q) {
                const float4 tq = *(const float4*)(tt + 4 * q);
                const float4 mq = *(const float4*)(mrow + ((q ^ (sq & 15)) << 2));
                float a[4] = {st + tq.x, st + tq.y, st + tq.z, st + tq.w};
                const float mk[4] = {mq.x, mq.y, mq.z, mq.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) a[k] = ex2_approx(mk[k] > 0.f ? fmaxf(a[k], kLeakySlope * a[k]) + ct : -INFINITY);
                put(q, make_float2(a[0], a[1]), make_float2(a[2], a[3]));
              }
            } else {
              const int qlo = qd & ~1;
              const float h0 = st + sRef[qlo * 4 + t], h1 = st + sRef[(qlo + 1) * 4 + t];
              const float2 A0 = make_float2(ex2_approx(h0 + ct), ex2_approx(h0 + ct));
              const float2 C0 = make_float2(ex2_approx(fmaf(kLeakySlope, h0, ct)), ex2_approx(fmaf(kLeakySlope, h0, ct)));
              const float2 A1 = make_float2(ex2_approx(h1 + ct), ex2_approx(h1 + ct));
              const float2 C1 = make_float2(ex2_approx(fmaf(kLeakySlope, h1, ct)), ex2_approx(fmaf(kLeakySlope, h1, ct)));
              const float* bd = sBD + t * 128;
#pragma unroll
              for (int q = 0; q < 16; ++q) {
                const float2 A = q < 8 ? A0 : A1, C = q < 8 ? C0 : C1;
                const float4 bq = *(const float4*)(bd + 4 * q), dq = *(const float4*)(bd + 64 + 4 * q);
                const float4 mq = *(const float4*)(mrow + ((q ^ (sq & 15)) << 2));
                const float2 ab01 = __fmul2_rn(A, make_float2(bq.x, bq.y)), ab23 = __fmul2_rn(A, make_float2(bq.z, bq.w));
                const float2 cd01 = __fmul2_rn(C, make_float2(dq.x, dq.y)), cd23 = __fmul2_rn(C, make_float2(dq.z, dq.w));
                const float2 e01 = __fmul2_rn(make_float2(fmaxf(ab01.x, cd01.x), fmaxf(ab01.y, cd01.y)), make_float2(mq.x, mq.y));
                const float2 e23 = __fmul2_rn(make_float2(fmaxf(ab23.x, cd23.x), fmaxf(ab23.y, cd23.y)), make_float2(mq.z, mq.w));
                put(q, e01, e23);
              }
            }
            // layer 0 reads the raw features: its Wh carries no log2(e) yet
            inv[t] = rcp_approx(z2.x + z2.y) * (l == 0 ? kLog2e : 1.f);
            // the group's e buffer is free once its previous gather completed
            if (t >= 1) wait_gather(t - 1);
            const uint32_t acol = tlane + kECol + (uint32_t)(32 * g);
#pragma unroll
            for (int k = 0; k < 4; ++k) tmem_st_x8(acol + 8 * k, *(const uint32_t(*)[8])(e2 + 8 * k));
            tmem_st_wait();
          }
          fence_proxy_async_smem();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&req[2 * g + b]);
          if (t >= 1) finish_head(t - 1);
        }
        wait_gather(3);
        finish_head(3);
        return true;
      };
      for (int l = 0; l < kLayers && ok; ++l, ++L) {
        const bool cont = l < kLayers - 1 ? layer(l, std::false_type{}) : layer(l, std::true_type{});
        if (!cont) break;
      }
      if (!ok) break;

      // ---------------- heads ----------------
      wok = mbar_wait(pol_full, pph & 1, abort_flag, kWaitLimitNs) && wok;
      ++pph;
      ok = epilogue_all(wok);  // also: value partial sums of both groups visible
      if (!ok) break;
      tc_fence_after();
      float* stage = (float*)(smem + kSmX);  // X is free once the policy MMA completed
      float* red = (float*)(smem + kSmRed);
      if (g == 0) {
        // policy: this square's 73 logits, softmax over the position's 4672
        float lgt[kPN];
        const uint32_t pcol = tlane + 128 * first_block(L);  // the block after the last layer's
        tmem_ld_x32(pcol, *(float(*)[32])(lgt));
        tmem_ld_x32(pcol + 32, *(float(*)[32])(lgt + 32));
        tmem_ld_x8(pcol + 64, *(float(*)[8])(lgt + 64));
        tmem_ld_x8(pcol + 72, *(float(*)[8])(lgt + 72));
        tmem_ld_wait();
        float mx = -INFINITY;
#pragma unroll
        for (int k = 0; k < kP; ++k) {
          lgt[k] += __ldg(p.w + ChOff::b_pi + k) * kLog2e;  // logits in base 2
          mx = fmaxf(mx, lgt[k]);
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) red[qd * 2] = mx;
        named_bar_sync(gbar, 128);
        mx = fmaxf(red[(qd & ~1) * 2], red[(qd | 1) * 2]);  // the two warps of this position
        float z = 0.f;
#pragma unroll
        for (int k = 0; k < kP; ++k) {
          lgt[k] = ex2_approx(lgt[k] - mx);
          z += lgt[k];
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
        if (lane == 0) red[qd * 2 + 1] = z;
        named_bar_sync(gbar, 128);
        const float iz = 1.0f / (red[(qd & ~1) * 2 + 1] + red[(qd | 1) * 2 + 1]);
        float* out = stage + pg * kA + sq * kP;
#pragma unroll
        for (int k = 0; k < kP; ++k) out[k] = lgt[k] * iz;
      } else if (warp - 4 < kGPT) {
        // value head of position (warp - 4): 64 hidden units, two per lane
        const int q2 = warp - 4, pos = tile * kGPT + q2;
        const float* zp = (const float*)(smem + kSmZ);
        float z0 = __ldg(p.w + ChOff::b_v1 + lane), z1 = __ldg(p.w + ChOff::b_v1 + 32 + lane);
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {  // [group][half]
          z0 += zp[(c4 * kGPT + q2) * 64 + lane];
          z1 += zp[(c4 * kGPT + q2) * 64 + 32 + lane];
        }
        float vv = fmaxf(z0, 0.f) * __ldg(p.w + ChOff::w_v2 + lane) + fmaxf(z1, 0.f) * __ldg(p.w + ChOff::w_v2 + 32 + lane);
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) vv += __shfl_xor_sync(0xffffffffu, vv, o);
        if (lane == 0 && pos < p.n) p.v[pos] = tanhf(vv + __ldg(p.w + ChOff::b_v2));
      }
      fence_proxy_async_smem();  // staged probabilities -> the bulk copy's async proxy
      tc_fence_before();
      named_bar_sync(1, kEpiWarps * 32);
      if (threadIdx.x == 0) {
        for (int q2 = 0; q2 < kGPT; ++q2) {
          const int pos = tile * kGPT + q2;
          if (pos < p.n) bulk_s2g(p.pi + (size_t)pos * kA, stage + q2 * kA, kA * 4);
        }
        bulk_commit();
        bulk_wait_read();  // X is rewritten by the next tile's encode
      }
      named_bar_sync(1, kEpiWarps * 32);
    }
    if (threadIdx.x == 0) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_flag && threadIdx.x == 0) atomicExch(p.err, 1);
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---- weight packing ----
// Chunks 0..28: per layer W_l^T (256 rows) + attention-score rows W_l a (16
// high parts, 16 remainders), [288 rows][64 K] swizzled; layer 0 has K = 18.
// Chunks 29..32: W_pi^T [80 rows (73 used)][64 K].
// Input feature of K index kk of X chunk c after layer 0: chunk c holds heads
// c (K 0-31) and c + 4 (K 32-63).
__host__ __device__ constexpr int x_feature(int c, int kk) { return kk < 32 ? 32 * c + kk : 32 * (c + 4) + kk - 32; }
// Output feature of projection row n: the first 128 rows are heads 0, 4, 1, 5
// and the second 128 heads 2, 6, 3, 7 (head_col's order inside a block).
__host__ __device__ constexpr int proj_feature(int n) {
  return 32 * (4 * ((n >> 5) & 1) + 2 * (n >> 7) + ((n >> 6) & 1)) + (n & 31);
}

template <typename OpT>
__global__ void pack_chess_kernel(const float* __restrict__ w, uint8_t* __restrict__ out) {
  const int chunk = blockIdx.x;
  if (chunk >= kLayerChunks) {
    const int c = chunk - kLayerChunks;
    uint8_t* dst = out + (size_t)kLayerChunks * kWChunk + (size_t)c * kPolChunk;
    for (int t = threadIdx.x; t < kPN * 64; t += blockDim.x) {
      const int n = t / 64, kk = t % 64, k = x_feature(c, kk);
      const size_t i = ChOff::w_pi + (size_t)k * kP + n;
      const float x = n < kP ? w[i] : 0.f;
      *(uint16_t*)(dst + sw128_offset(n, kk)) = weight_bits_sr<OpT>(x, (uint32_t)i);
    }
    return;
  }
  const int layer = chunk == 0 ? 0 : 1 + (chunk - 1) / 4;
  const int c = chunk == 0 ? 0 : (chunk - 1) % 4;
  const int fin = layer == 0 ? kF : 256;
  const float* W = w + ChOff::W(layer);
  const float* A = w + ChOff::a(layer);
  uint8_t* dst = out + (size_t)chunk * kWChunk;
  for (int t = threadIdx.x; t < 256 * 64; t += blockDim.x) {
    const int n = t / 64, kk = t % 64, k = layer == 0 ? kk : x_feature(c, kk);
    const size_t i = (size_t)k * 256 + proj_feature(n);
    const float x = k < fin ? W[i] : 0.f;
    *(uint16_t*)(dst + sw128_offset(n, kk)) = weight_bits_sr<OpT>(x, (uint32_t)(ChOff::W(layer) + i));
  }
  for (int t = threadIdx.x; t < 16 * 64; t += blockDim.x) {
    const int j = t / 64, kk = t % 64, k = layer == 0 ? kk : x_feature(c, kk), h = j >> 1, v = j & 1;
    float acc = 0.f;
    if (k < fin)
      for (int f = 0; f < 32; ++f) acc = fmaf(W[(size_t)k * 256 + 32 * h + f], A[(2 * h + v) * 32 + f], acc);
    if (layer == 0) acc *= kLog2e;  // layer 0's scores in base 2, like the later layers'
    const float hi = OpType<OpT>::round(acc);
    *(uint16_t*)(dst + sw128_offset(256 + j, kk)) = OpType<OpT>::bits(hi);
    *(uint16_t*)(dst + sw128_offset(272 + j, kk)) = OpType<OpT>::bits(acc - hi);
  }
}

}  // namespace

size_t chess_tc_packed_bytes() { return (size_t)kLayerChunks * kWChunk + 4 * (size_t)kPolChunk; }

cudaError_t launch_chess_tc_pack(int fp16, const float* d_weights, void* d_packed, cudaStream_t stream) {
  if (fp16) pack_chess_kernel<__half><<<kChunksPerTile, 256, 0, stream>>>(d_weights, (uint8_t*)d_packed);
  else pack_chess_kernel<__nv_bfloat16><<<kChunksPerTile, 256, 0, stream>>>(d_weights, (uint8_t*)d_packed);
  return cudaGetLastError();
}

cudaError_t launch_chess_tc(int fp16, const void* d_packed, const float* d_weights, const int8_t* d_boards,
                            const int8_t* d_side, int n, float* d_pi, float* d_v, int* d_err, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  if (((uintptr_t)d_pi & 15u) != 0) return cudaErrorInvalidValue;  // bulk stores of the policy rows
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
  const char* gap = getenv("GZ_CHESS_FACTOR_GAP");
  p.max_gap = gap && *gap ? (float)atof(gap) : kMaxFactorGap;
  if (!(p.max_gap <= kMaxFactorGap)) p.max_gap = kMaxFactorGap;  // larger gaps would leave the fp32 range
  auto kern = fp16 ? gat_tc_chess_kernel<__half> : gat_tc_chess_kernel<__nv_bfloat16>;
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
  const int grid = full_grid < p.num_tiles ? full_grid : p.num_tiles;
  kern<<<grid, kThreads, kSmemBytes, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace gz
