// Tensor-core (tcgen05) Connect4 ResNet forward: stem, 10 residual blocks
// and both heads in one persistent launch, one CTA per SM.
//
// A tile is 128 rows = 3 positions x 42 squares (+2 padding rows); the
// activations of the tile stay in shared memory for all 21 convolutions.
// A 3x3 convolution is an implicit GEMM over 9 taps:
//     out[p][co] = sum_t sum_ci X[p + s_t][ci] W_t[co][ci],
// s_t = 7 dy + dx the row shift of tap t inside the row-major board.  The
// activation tile is K-major in the 128-byte swizzle with 128-byte rows, so
// the shifted operand of a tap is the same tile viewed from a start address
// s_t rows further (the swizzle follows the absolute address, so the view
// needs no other change); 8 guard rows on either side keep every view inside
// the buffer.
// Squares whose tap falls off the board (and the padding rows) are excluded
// with the MMA's per-row disable mask, which is exactly zero padding.  The
// centre tap runs first with accumulation off, so every real row is
// initialised.  BN is folded into a per-channel scale and shift; the
// epilogue applies scale/shift, the residual add and ReLU in fp32 and writes
// the next layer's bf16 tile.  The last epilogue also computes the 1x1
// head convolutions, and the heads (FC 84->7 softmax, FC 42->128 ReLU ->1
// tanh) finish in fp32.
//
// Two tiles are in flight per CTA (slots A and B, each with its own
// activations and tensor-memory accumulator): the MMAs of one slot's
// convolution run while the epilogue warps finish the other slot's, so the
// tensor pipe does not idle during the epilogues.
//
// Reference: networks/resnet/resnet.cu:506-667 (forward_resnet; the
// reference's residual "add" overwrites, resnet.cu:588-591, and its BN runs
// in training mode; here BN is in inference form and the add is real).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "gz_games.h"
#include "gz_internal.h"
#include "gz_round.h"
#include "gz_sm100.h"

namespace gz {
namespace {

using namespace sm100;

constexpr int kN = 42;
constexpr int kGPT = 3;
constexpr int kRows = 128;
constexpr int kC = kResChannels;          // 128
constexpr int kConvs = 1 + 2 * kResBlocks;  // 21
constexpr int kEpiWarps = 8;                // row quarter x channel half
constexpr int kThreads = (kEpiWarps + 2) * 32;
constexpr int kProducerWarp = kEpiWarps;
constexpr int kMmaWarp = kEpiWarps + 1;
constexpr int kWChunk = 16384;              // 128 co rows x 64 ci x 2 B
constexpr int kChunksPerTile = 9 + (kConvs - 1) * 18;
// The ring moves one tap (both 64-channel chunks, 32 KB) per copy, three
// slots deep: two taps' copies are in flight while the MMAs of the current
// one run.  Measured on B200: 32 KB bulk copies stream about 77 bytes per
// cycle per SM from L2 against 45 for 16 KB copies, and a tile's tower
// needs about 62 (the weights are re-streamed for every tile); two 32 KB
// slots exposed a copy's latency at every tap, four 16 KB slots its
// bandwidth.
constexpr int kWSlot = 2 * kWChunk;
constexpr int kWSlots = 3;
constexpr uint32_t kTmemCols = 256;         // slot s accumulates in columns [128 s, 128 s + 128)
constexpr uint64_t kWaitLimitNs = 4000000000ull;
constexpr int kActChunk = kRows * 128;      // one 64-channel K chunk, 16 KB
constexpr int kActBytes = 2 * kActChunk;    // 128 channels

// Shared memory map.  The folded BN parameters, barriers and the like come
// first; then the activations, slot s's at kSmAct + s * kSlotBytes, back to
// back; then the weight ring.  A tap's shifted view of a buffer starts up to
// 8 rows before its first row or ends up to 8 rows after its last: those
// rows belong to the neighbouring buffer (or to the regions before and after
// the activations) and feed only output rows the tap's mask disables, so
// the buffers need no guard rows.
constexpr int kSmBn = 0;                          // [2 parity][scale 128, shift 128]
constexpr int kSmBar = kSmBn + 2 * 2 * kC * 4;
constexpr int kNumBars = 2 * kWSlots + 5;         // full, empty, acc_full[2], act_ready[2], drain
constexpr int kSmMisc = kSmBar + kNumBars * 8;
constexpr int kSmAct = 3072;
constexpr int kSmA0 = 0;                          // block input / residual (offsets inside a slot)
constexpr int kSmA1 = kSmA0 + kActBytes;          // intermediate (and the stem input)
constexpr int kSlotBytes = 2 * kActBytes;
constexpr int kSmW = kSmAct + 2 * kSlotBytes;     // weight ring
constexpr int kSmemBytes = kSmW + kWSlots * kWSlot;
// Head scratch during the last convolution's epilogue, inside the slot's A1
// buffer (that convolution's input, dead once its accumulator is complete).
constexpr int kHdHead = 0;                          // [2 halves][128 rows][3] partial head dots
constexpr int kHdFeat = kHdHead + 2 * kRows * 3 * 4;  // [3 pos][84 policy + 42 value] features
constexpr int kHdHid = kHdFeat + kGPT * 128 * 4;    // [3][128] value hidden
constexpr int kHdLogit = kHdHid + kGPT * 128 * 4;   // [3][8]
static_assert(kHdLogit + kGPT * 8 * 4 <= kActBytes, "head scratch fits in an activation buffer");
static_assert(kSmMisc + 16 <= kSmAct, "header region");
static_assert(kSmAct >= 1024, "room before the first buffer for a tap's 8-row lead");
static_assert(kSmAct % 1024 == 0 && kSmW % 1024 == 0 && kActChunk % 1024 == 0, "swizzle alignment");
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");

// Packed layout (bytes) after the weight chunks: per conv, scale[128] and
// shift[128] (fp32, BN folded).
constexpr size_t kPackedW = (size_t)kChunksPerTile * kWChunk;
constexpr size_t kPackedBytes = kPackedW + (size_t)kConvs * 2 * kC * 4;

// Tap order: centre first (initialises every real row), then the others.
__host__ __device__ constexpr int tap_dy(int t) { return t == 0 ? 0 : ((t <= 4 ? t - 1 : t) / 3) - 1; }
__host__ __device__ constexpr int tap_dx(int t) { return t == 0 ? 0 : ((t <= 4 ? t - 1 : t) % 3) - 1; }

// Per-tap row masks (bit set = row skipped): rows whose tap leaves the board,
// and the two padding rows.  Identical for every tile; built at compile time
// so the MMA loop reads them as immediates.
struct TapMasks {
  uint32_t m[9][4];
};
__host__ __device__ constexpr TapMasks tap_masks() {
  TapMasks k{};
  for (int t = 0; t < 9; ++t)
    for (int r = 0; r < kRows; ++r) {
      const int li = r % kN, rr = li / 7 + tap_dy(t), cc = li % 7 + tap_dx(t);
      const bool live = r < kGPT * kN && rr >= 0 && rr < 6 && cc >= 0 && cc < 7;
      if (!live) k.m[t][r >> 5] |= 1u << (r & 31);
    }
  return k;
}

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

// Operand type of the convolutions: bf16 (default) or fp16.
template <typename T> struct ResOp;
template <> struct ResOp<__nv_bfloat16> {
  static constexpr uint32_t fmt = 1;
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  static __device__ __forceinline__ float2 unpack(uint32_t w) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
  }
  static __device__ __forceinline__ uint16_t bits(float x) { return __bfloat16_as_ushort(__float2bfloat16_rn(x)); }
};
template <> struct ResOp<__half> {
  static constexpr uint32_t fmt = 0;
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  static __device__ __forceinline__ float2 unpack(uint32_t w) {
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
  }
  static __device__ __forceinline__ uint16_t bits(float x) { return __half_as_ushort(__float2half_rn(x)); }
};

struct ResParams {
  const uint8_t* packed;
  const float* w;  // fp32 blob (head weights)
  const int8_t* boards;
  const int8_t* side;
  float* pi;
  float* v;
  int* err;
  int n;
  int num_tiles;
};

template <typename OpT>
__global__ void __launch_bounds__(kThreads, 1) resnet_tc_kernel(ResParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) atomicExch(p.err, 2);
    return;
  }
  uint64_t* bars = (uint64_t*)(smem + kSmBar);
  uint64_t* full = bars;
  uint64_t* empty = bars + kWSlots;
  uint64_t* acc_full = bars + 2 * kWSlots;  // [slot]
  uint64_t* act_ready = acc_full + 2;       // [slot]
  uint64_t* drain = acc_full + 4;
  uint32_t* tmem_slot = (uint32_t*)(smem + kSmMisc);
  volatile int* abort_flag = (volatile int*)(smem + kSmMisc + 4);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const ResLayout RL = res_layout();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kWSlots; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int sl = 0; sl < 2; ++sl) {
      mbar_init(&acc_full[sl], 1);
      mbar_init(&act_ready[sl], kEpiWarps);
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
    if (lane == 0) {
      uint32_t q = 0;
      bool ok = true;
      // consumption order: per tile pair, per conv, slot A's nine taps then slot B's
      for (int ta = blockIdx.x; ta < p.num_tiles && ok; ta += 2 * gridDim.x)
        for (int u = 0; u < 18 * kConvs && ok; ++u, ++q) {
          const int cv = u / 18, t = u % 9;
          // stem tap: one 16 KB chunk; block conv tap: its two adjacent chunks in one copy
          const int c = cv == 0 ? t : 9 + (cv - 1) * 18 + 2 * t;
          const uint32_t bytes = cv == 0 ? kWChunk : 2 * kWChunk;
          const int s = q % kWSlots;
          ok = mbar_wait(&empty[s], ((q / kWSlots) & 1) ^ 1, abort_flag, kWaitLimitNs);
          if (!ok) break;
          mbar_arrive_expect_tx(&full[s], bytes);
          bulk_g2s(smem + kSmW + s * kWSlot, p.packed + (size_t)c * kWChunk, bytes, &full[s]);
        }
      for (uint32_t k = (q > kWSlots ? q - kWSlots : 0); k < q; ++k)
        mbar_wait(&full[k % kWSlots], (k / kWSlots) & 1, abort_flag, kWaitLimitNs);
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      constexpr TapMasks kMask = tap_masks();
      constexpr uint32_t idesc = idesc_f16(ResOp<OpT>::fmt, 128, 128);
      uint32_t q = 0, aph[2] = {0, 0};
      bool ok = true;
      for (int ta = blockIdx.x; ta < p.num_tiles && ok; ta += 2 * gridDim.x) {
        for (int u = 0; u < 2 * kConvs && ok; ++u) {
          const int cv = u >> 1, sl = u & 1;
          ok = mbar_wait(&act_ready[sl], aph[sl] & 1, abort_flag, kWaitLimitNs);
          ++aph[sl];
          if (!ok) break;
          tc_fence_after();
          const uint32_t dt = tmem + (uint32_t)(128 * sl);
          // input buffer: stem reads A1 (input planes), block conv1 reads A0, conv2 reads A1
          const uint32_t in = smem_u32(smem + kSmAct + sl * kSlotBytes + ((cv == 0 || (cv & 1) == 0) ? kSmA1 : kSmA0));
          const int nchunk = cv == 0 ? 1 : 2;
          // One thread issues every MMA, so its own instruction stream bounds
          // the MMA rate: the taps are unrolled (masks stay in registers) and
          // descriptors advance by adding (byte offset >> 4) to the start
          // address field (shared addresses stay below 2^18: no carry).
          const uint64_t in_desc = sw128_desc_shifted(in);
          const uint64_t w_desc = sw128_desc(smem_u32(smem + kSmW));
#pragma unroll
          for (int t = 0; t < 9; ++t) {
            const int shift = 7 * tap_dy(t) + tap_dx(t);  // rows; x 128 bytes
            if (!ok) break;
            const int s = q % kWSlots;  // this tap's weights: one slot
            ok = mbar_wait(&full[s], (q / kWSlots) & 1, abort_flag, kWaitLimitNs);
            ++q;
            if (!ok) break;
            tc_fence_after();
            for (int c = 0; c < nchunk; ++c) {  // 64-channel K chunks of this tap
              const uint64_t wd = w_desc + (uint64_t)((s * kWSlot + c * kWChunk) >> 4);
              const uint64_t ad = in_desc + (uint64_t)((c * kActChunk + shift * 128) >> 4);
              mma_f16_ss_masked(dt, ad, wd, idesc, (t | c) != 0, kMask.m[t]);
              if (cv != 0) {
#pragma unroll
                for (int kk = 1; kk < 4; ++kk) mma_f16_ss_masked(dt, ad + kk * 2, wd + kk * 2, idesc, 1, kMask.m[t]);
              }
            }
            mma_commit(&empty[s]);
          }
          if (ok) mma_commit(&acc_full[sl]);
        }
      }
      mma_commit(drain);
      mbar_wait(drain, 0, abort_flag, kWaitLimitNs);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue: warp = (row quarter qd, channel half hf) ----------------
    const int qd = warp & 3, hf = warp >> 2;
    const int r = 32 * qd + lane;  // tile row of this thread
    const uint32_t tlane = tmem + ((uint32_t)(32 * qd) << 16);
    const float* bnp = (const float*)(p.packed + kPackedW);
    uint32_t accph[2] = {0, 0};
    bool ok = true;
    for (int ta = blockIdx.x; ta < p.num_tiles && ok; ta += 2 * gridDim.x) {
      // slot sl holds tile ta + sl * gridDim.x (past the last tile: zero
      // inputs, outputs never written since its positions are >= n)
      for (int sl = 0; sl < 2; ++sl) {
        const int tile = ta + sl * (int)gridDim.x;
        // -- stem input: 3 planes (own, opponent, first-player-to-move) in A1 chunk 0 --
        const int g = r / kN, li = r % kN, pos = tile * kGPT + g;
        float f0 = 0.f, f1 = 0.f, f2 = 0.f;
        if (g < kGPT && pos < p.n) {
          const int sd = p.side[pos], b = p.boards[(size_t)pos * 42 + li];
          f0 = b == sd ? 1.f : 0.f;
          f1 = b == -sd ? 1.f : 0.f;
          f2 = sd == 1 ? 1.f : 0.f;
        }
        if (hf == 0) {
          uint8_t* row = smem + kSmAct + sl * kSlotBytes + kSmA1 + r * 128;
          const int rs = r & 7;
          *(uint4*)(row + ((0 ^ rs) << 4)) = make_uint4(ResOp<OpT>::pack(f0, f1), ResOp<OpT>::pack(f2, 0.f), 0u, 0u);
          *(uint4*)(row + ((1 ^ rs) << 4)) = make_uint4(0u, 0u, 0u, 0u);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&act_ready[sl]);
      }

      for (int u = 0; u < 2 * kConvs && ok; ++u) {
        const int cv = u >> 1, sl = u & 1, tile = ta + sl * (int)gridDim.x;
        // folded BN of this conv into shared memory (by parity; both slots use it)
        float* bn = (float*)(smem + kSmBn) + (cv & 1) * 2 * kC;
        if (sl == 0)
          for (int t = threadIdx.x; t < 2 * kC; t += kEpiWarps * 32) bn[t] = __ldg(bnp + (size_t)cv * 2 * kC + t);
        ok = epilogue_all(mbar_wait(&acc_full[sl], accph[sl] & 1, abort_flag, kWaitLimitNs));
        ++accph[sl];
        if (!ok) break;
        tc_fence_after();
        uint8_t* const sbase = smem + kSmAct + sl * kSlotBytes;
        const uint32_t tslot = tlane + (uint32_t)(128 * sl);
        const bool second = cv > 0 && (cv & 1) == 0;  // second conv of a block: residual add
        const bool last = cv == kConvs - 1;
        // output: stem and conv2 -> A0, conv1 -> A1
        uint8_t* outb = sbase + ((cv == 0 || second) ? kSmA0 : kSmA1);
        float hp0 = 0.f, hp1 = 0.f, hv = 0.f;  // partial 1x1 head convolutions (last conv)
#pragma unroll 1
        for (int cb = 0; cb < 2; ++cb) {  // 32-channel blocks of this half
          const int c0 = 64 * hf + 32 * cb;
          float acc[32];
          tmem_ld_x32(tslot + (uint32_t)c0, acc);
          tmem_ld_wait();
          const float4* sc4 = (const float4*)(bn + c0);
          const float4* sh4 = (const float4*)(bn + kC + c0);
          float y[32];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const float4 sc = sc4[k], sh = sh4[k];
            y[4 * k + 0] = fmaf(acc[4 * k + 0], sc.x, sh.x);
            y[4 * k + 1] = fmaf(acc[4 * k + 1], sc.y, sh.y);
            y[4 * k + 2] = fmaf(acc[4 * k + 2], sc.z, sh.z);
            y[4 * k + 3] = fmaf(acc[4 * k + 3], sc.w, sh.w);
          }
          // row r, channels c0..c0+31: K chunk c0/64, 16-byte units (c0%64)/8 + u
          const int rs = r & 7;
          uint8_t* orow = outb + (c0 >> 6) * kActChunk + r * 128;
          const uint8_t* rrow = sbase + kSmA0 + (c0 >> 6) * kActChunk + r * 128;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int unit = ((((c0 & 63) >> 3) + u) ^ rs) << 4;
            if (second) {
              const uint4 res = *(const uint4*)(rrow + unit);
              const uint32_t rv[4] = {res.x, res.y, res.z, res.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 f = ResOp<OpT>::unpack(rv[e]);
                y[8 * u + 2 * e] += f.x;
                y[8 * u + 2 * e + 1] += f.y;
              }
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) y[8 * u + e] = fmaxf(y[8 * u + e], 0.f);
            if (!last)
              *(uint4*)(orow + unit) =
                  make_uint4(ResOp<OpT>::pack(y[8 * u], y[8 * u + 1]), ResOp<OpT>::pack(y[8 * u + 2], y[8 * u + 3]),
                             ResOp<OpT>::pack(y[8 * u + 4], y[8 * u + 5]), ResOp<OpT>::pack(y[8 * u + 6], y[8 * u + 7]));
          }
          if (last) {
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              hp0 = fmaf(y[e], __ldg(p.w + RL.pol_w + c0 + e), hp0);
              hp1 = fmaf(y[e], __ldg(p.w + RL.pol_w + kC + c0 + e), hp1);
              hv = fmaf(y[e], __ldg(p.w + RL.val_w + c0 + e), hv);
            }
          }
        }
        if (!last) {
          fence_proxy_async_smem();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&act_ready[sl]);
          continue;
        }
        // ---------------- heads (fp32) ----------------
        tc_fence_before();
        float* part = (float*)(sbase + kSmA1 + kHdHead);
        part[(hf * kRows + r) * 3 + 0] = hp0;
        part[(hf * kRows + r) * 3 + 1] = hp1;
        part[(hf * kRows + r) * 3 + 2] = hv;
        named_bar_sync(1, kEpiWarps * 32);
        float* feat = (float*)(sbase + kSmA1 + kHdFeat);  // [3][128]: 84 policy, 42 value
        const int tid = threadIdx.x;
        if (tid < kGPT * kN) {
          const int g = tid / kN, li = tid % kN, row = tid;
          const float* pb = p.w + RL.pol_bn;  // gamma, beta, mean, var (2 channels each)
          const float* vb = p.w + RL.val_bn;
          for (int ch = 0; ch < 2; ++ch) {
            const float x = part[row * 3 + ch] + part[(kRows + row) * 3 + ch];
            const float sc = __ldg(pb + ch) / sqrtf(__ldg(pb + 6 + ch) + kBnEps);
            feat[g * 128 + ch * kN + li] = (x - __ldg(pb + 4 + ch)) * sc + __ldg(pb + 2 + ch);
          }
          const float x = part[row * 3 + 2] + part[(kRows + row) * 3 + 2];
          const float sc = __ldg(vb + 0) / sqrtf(__ldg(vb + 3) + kBnEps);
          feat[g * 128 + 84 + li] = (x - __ldg(vb + 2)) * sc + __ldg(vb + 1);
        }
        named_bar_sync(1, kEpiWarps * 32);
        float* hid = (float*)(sbase + kSmA1 + kHdHid);
        float* logit = (float*)(sbase + kSmA1 + kHdLogit);
        for (int t = tid; t < kGPT * kResValueHidden; t += kEpiWarps * 32) {
          const int g = t / kResValueHidden, u = t % kResValueHidden;
          float a = __ldg(p.w + RL.val_fc1_b + u);
          for (int i = 0; i < kN; ++i) a = fmaf(feat[g * 128 + 84 + i], __ldg(p.w + RL.val_fc1 + i * kResValueHidden + u), a);
          hid[g * 128 + u] = fmaxf(a, 0.f);
        }
        if (tid >= 192 && tid < 192 + kGPT * 7) {
          const int k = tid - 192, g = k / 7, j = k % 7;
          float a = __ldg(p.w + RL.pol_fc_b + j);
          for (int i = 0; i < 84; ++i) a = fmaf(feat[g * 128 + i], __ldg(p.w + RL.pol_fc + i * 7 + j), a);
          logit[g * 8 + j] = a;
        }
        named_bar_sync(1, kEpiWarps * 32);
        if (warp < kGPT) {
          const int g = warp, pos = tile * kGPT + g;
          float vv = 0.f;
          for (int u = lane; u < kResValueHidden; u += 32) vv = fmaf(hid[g * 128 + u], __ldg(p.w + RL.val_fc2 + u), vv);
#pragma unroll
          for (int o = 16; o >= 1; o >>= 1) vv += __shfl_xor_sync(0xffffffffu, vv, o);
          const float lg = lane < 7 ? logit[g * 8 + lane] : -INFINITY;
          float mx = lg;
#pragma unroll
          for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
          const float ex = lane < 7 ? expf(lg - mx) : 0.f;
          float z = ex;
#pragma unroll
          for (int o = 16; o >= 1; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
          if (pos < p.n) {
            if (lane < 7) p.pi[(size_t)pos * 7 + lane] = ex / z;
            if (lane == 0) p.v[pos] = tanhf(vv + __ldg(p.w + RL.val_fc2_b));
          }
        }
        named_bar_sync(1, kEpiWarps * 32);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (*abort_flag && threadIdx.x == 0) atomicExch(p.err, 1);
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// Pack: per conv, per tap (centre first), per 64-channel K chunk: W_t^T as a
// [128 co][64 ci] bf16 tile in the 128-byte swizzle; then folded BN.
template <typename OpT>
__global__ void pack_resnet_kernel(const float* __restrict__ w, uint8_t* __restrict__ out) {
  const ResLayout RL = res_layout();
  const int chunk = blockIdx.x;
  int cv, t, c;
  if (chunk < 9) {
    cv = 0; t = chunk; c = 0;
  } else {
    cv = 1 + (chunk - 9) / 18;
    t = ((chunk - 9) % 18) / 2;
    c = (chunk - 9) % 2;
  }
  const int cin = cv == 0 ? kResInPlanes : kC;
  const size_t wbase = cv == 0 ? RL.stem_w : (cv & 1) ? RL.conv1_w[(cv - 1) / 2] : RL.conv2_w[(cv - 1) / 2];
  const float* W = w + wbase;
  const int ky = tap_dy(t) + 1, kx = tap_dx(t) + 1;
  uint8_t* dst = out + (size_t)chunk * kWChunk;
  for (int i = threadIdx.x; i < 128 * 64; i += blockDim.x) {
    const int co = i / 64, kk = i % 64, ci = c * 64 + kk;
    const size_t e = (((size_t)co * 3 + ky) * 3 + kx) * cin + ci;
    const float x = ci < cin ? W[e] : 0.f;
    *(uint16_t*)(dst + sw128_offset(co, kk)) = weight_bits_sr<OpT>(x, (uint32_t)(wbase + e));
  }
  if (chunk < kConvs) {  // folded BN of conv `chunk`
    const int k = chunk;
    const float* bn = w + (k == 0 ? RL.stem_bn : (k & 1) ? RL.bn1[(k - 1) / 2] : RL.bn2[(k - 1) / 2]);
    float* o = (float*)(out + kPackedW) + (size_t)k * 2 * kC;
    for (int co = threadIdx.x; co < kC; co += blockDim.x) {
      const float sc = bn[co] / sqrtf(bn[3 * kC + co] + kBnEps);
      o[co] = sc;
      o[kC + co] = bn[kC + co] - bn[2 * kC + co] * sc;
    }
  }
}

}  // namespace

size_t resnet_tc_packed_bytes() { return kPackedBytes; }

cudaError_t launch_resnet_tc_pack(int fp16, const float* d_weights, void* d_packed, cudaStream_t stream) {
  if (fp16) pack_resnet_kernel<__half><<<kChunksPerTile, 256, 0, stream>>>(d_weights, (uint8_t*)d_packed);
  else pack_resnet_kernel<__nv_bfloat16><<<kChunksPerTile, 256, 0, stream>>>(d_weights, (uint8_t*)d_packed);
  return cudaGetLastError();
}

cudaError_t launch_resnet_tc(int fp16, const void* d_packed, const float* d_weights, const int8_t* d_boards,
                             const int8_t* d_side, int n, float* d_pi, float* d_v, int* d_err, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  ResParams p;
  p.packed = (const uint8_t*)d_packed;
  p.w = d_weights;
  p.boards = d_boards;
  p.side = d_side;
  p.pi = d_pi;
  p.v = d_v;
  p.err = d_err;
  p.n = n;
  p.num_tiles = (n + kGPT - 1) / kGPT;
  auto kern = fp16 ? resnet_tc_kernel<__half> : resnet_tc_kernel<__nv_bfloat16>;
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
