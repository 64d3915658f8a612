// Tensor-core (tcgen05) GAT forward for Connect4: all six layers and both
// heads in one persistent launch.
//
// Layout of one tile: 128 node columns = 3 positions x 42 nodes (+2 padding).
// Each layer computes the projection transposed,
//     Wh^T[256 features][128 nodes] = W^T[256][K] . X^T[K][128],
// as two M = 128 halves with tcgen05.mma (bf16 or fp16 operands, fp32
// accumulators in tensor memory).  Tensor memory then holds one feature per
// lane and one node per column, so epilogue warp w owns head w (32
// features, one per lane) for every node of the tile, and the per-edge stage
// runs in registers:
//   scores   s_i = a_self . Wh_i, t_j = a_nbr . Wh_j  (warp-shuffle
//            transpose-reductions across the 32 feature lanes)
//   softmax  alpha_ij = softmax_j LeakyReLU_0.2(s_i + t_j) over the static
//            Connect4 CSR (computed once per head, kept in shared memory)
//   gather   out_i = sum_j alpha_ij Wh_j, fully unrolled over the CSR with
//            Wh_j in registers
//   bias, ELU, and the bf16 / fp16 store of X_{l+1} into the 128-byte
//   swizzled shared-memory tile the next projection reads.
// The last layer feeds the value head (mean-pool, 256->64 ReLU, 64->1 tanh)
// and the column-pooled policy head in fp32 instead of storing X.
//
// Weights W_l^T are pre-packed on the device into 16 KB chunks (128 feature
// rows x 64 K, 128-byte swizzled, bf16/fp16) and streamed into a ring of
// shared-memory slots by one producer thread with 1-D bulk async copies
// (TMA engine); one thread issues the MMAs.  Two CTAs share an SM so one's
// projection overlaps the other's edge stage.
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
#include "gz_sm100.h"

namespace gz {
namespace {

using namespace sm100;

constexpr int kN = 42;             // Connect4 nodes
constexpr int kGPT = 3;            // positions per tile
constexpr int kTileCols = 128;     // node columns per tile (MMA N)
constexpr int kLayers = 6;
constexpr int kChunkBytes = 16384; // 128 rows x 64 K x 2 B
constexpr int kSlots = 2;
constexpr int kEpiWarps = 8;
constexpr int kThreads = (kEpiWarps + 2) * 32;
constexpr int kProducerWarp = kEpiWarps;
constexpr int kMmaWarp = kEpiWarps + 1;
constexpr int kTmemCols = 256;     // two M-halves x 128 node columns, fp32
constexpr uint64_t kWaitLimitNs = 4000000000ull;  // 4 s per wait
constexpr int kChunksPerTile = 2 + (kLayers - 1) * 8;

// Static Connect4 board graph (8-neighbourhood + self, ascending).
struct C4Graph {
  int rp[kN + 1];
  int col[304];
};
constexpr C4Graph make_c4_graph() {
  C4Graph g{};
  int n = 0;
  for (int i = 0; i < kN; ++i) {
    g.rp[i] = n;
    for (int j = 0; j < kN; ++j) {
      int dr = j / 7 - i / 7, dc = j % 7 - i % 7;
      if (dr >= -1 && dr <= 1 && dc >= -1 && dc <= 1) g.col[n++] = j;
    }
  }
  g.rp[kN] = n;
  return g;
}
constexpr C4Graph kC4 = make_c4_graph();
static_assert(kC4.rp[kN] == 304, "Connect4 graph has 304 directed edges incl. self loops");

// Compile-time views of the graph for the fully unrolled gather.
template <int E> struct EdgeCol { static constexpr int value = kC4.col[E]; };
template <int I> struct RowPtr { static constexpr int value = kC4.rp[I]; };

__constant__ int c_rp[kN + 1];
__constant__ int c_col[304];

// acc += sum over edges E in [E0, E1) of alpha[E] * wh[col(E)]; alpha read as
// float4 words (shared memory, 16-byte aligned).
template <int E, int E1>
__device__ __forceinline__ void gather_edges(float& acc, const float (&wh)[kN], const float4* a4) {
  if constexpr (E < E1) {
    const float4 w4 = a4[E >> 2];
    const float ae = (E & 3) == 0 ? w4.x : (E & 3) == 1 ? w4.y : (E & 3) == 2 ? w4.z : w4.w;
    acc = fmaf(ae, wh[EdgeCol<E>::value], acc);
    gather_edges<E + 1, E1>(acc, wh, a4);
  }
}

// For every node I: out_I = sum_j alpha_Ij wh_j, then fin(I, out_I) with I as
// a compile-time constant.
template <int I, typename Fin>
__device__ __forceinline__ void gather_rows(const float (&wh)[kN], const float4* a4, Fin&& fin) {
  if constexpr (I < kN) {
    float acc = 0.f;
    gather_edges<RowPtr<I>::value, RowPtr<I + 1>::value>(acc, wh, a4);
    fin(std::integral_constant<int, I>{}, acc);
    gather_rows<I + 1>(wh, a4, fin);
  }
}

// Shared memory map (bytes).
constexpr int kSmX = 0;                                  // 4 chunks: X tile, K-major swizzled
constexpr int kSmW = kSmX + 4 * kChunkBytes;             // weight ring
constexpr int kWarpScratchFloats = 48 + 48 + 48 + 304;   // s_self, s_nbr, 1/z, alpha (16-byte aligned parts)
constexpr int kSmScratch = kSmW + kSlots * kChunkBytes;
constexpr int kSmRp = kSmScratch + kEpiWarps * kWarpScratchFloats * 4;  // CSR row pointers [43]
constexpr int kSmBar = kSmRp + 48 * 4;
constexpr int kNumBars = 2 * kSlots + 3;                 // full[], empty[], acc_full, x_ready, drain
constexpr int kSmMisc = kSmBar + kNumBars * 8;           // tmem base, abort flag
constexpr int kSmemBytes = kSmMisc + 16;
constexpr int kSmemAlloc = kSmemBytes;                    // base must be 1024-aligned (checked)
static_assert(kSmemAlloc <= 113 * 1024, "two CTAs per SM");

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
};
template <> struct OpType<__half> {
  static constexpr uint32_t fmt = 0;
  static __device__ __forceinline__ uint16_t bits(float x) { return __half_as_ushort(__float2half_rn(x)); }
};

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Barrier over the epilogue warps that also ANDs `ok` across them, so they
// continue or give up together (no warp is left waiting in a later barrier).
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

// Sum over the 32 lanes of a * x[B + k] for k < 32 (a reduce-scatter across
// lanes); lane l ends with the sum for k = l.
template <int B, int NX>
__device__ __forceinline__ float dot_scatter32(const float (&x)[NX], float a, int lane) {
  float v[16];
  const bool up16 = lane & 16;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const float lo = a * x[B + k], hi = a * x[B + k + 16];
    v[k] = (up16 ? hi : lo) + __shfl_xor_sync(0xffffffffu, up16 ? lo : hi, 16);
  }
#pragma unroll
  for (int o = 8; o >= 1; o >>= 1) {
    const bool up = lane & o;
#pragma unroll
    for (int k = 0; k < o; ++k) {
      float send = up ? v[k] : v[k + o];
      float keep = up ? v[k + o] : v[k];
      v[k] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  return v[0];
}

// Sum over the 32 lanes of a * x[B + k] for k < 16 (entries at or past NX
// count as 0); lane l ends with the sum for k = l & 15.
template <int B, int NX>
__device__ __forceinline__ float dot_scatter16(const float (&x)[NX], float a, int lane) {
  float v[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    v[k] = B + k < NX ? a * x[B + k < NX ? B + k : 0] : 0.f;
    v[k] += __shfl_xor_sync(0xffffffffu, v[k], 16);
  }
#pragma unroll
  for (int o = 8; o >= 1; o >>= 1) {
    const bool up = lane & o;
#pragma unroll
    for (int k = 0; k < o; ++k) {
      float send = up ? v[k] : v[k + o];
      float keep = up ? v[k + o] : v[k];
      v[k] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  return v[0];
}

__device__ __forceinline__ float lrelu(float x) { return x > 0.f ? x : kLeakySlope * x; }
__device__ __forceinline__ float elu_fast(float x) { return x > 0.f ? x : __expf(x) - 1.0f; }

template <int OFF>
__device__ __forceinline__ void st_shared_u16(uint32_t addr, uint16_t v) {
  asm volatile("st.shared.b16 [%0+%1], %2;" ::"r"(addr), "n"(OFF), "h"(v) : "memory");
}

template <int I>
__device__ __forceinline__ float pick4(const float4* a4) {
  const float4 w4 = a4[I >> 2];
  return (I & 3) == 0 ? w4.x : (I & 3) == 1 ? w4.y : (I & 3) == 2 ? w4.z : w4.w;
}

// Epilogue of one position (compile-time slot G_ of the tile) for the head
// owned by this warp: scores, neighbour softmax, gather, bias + ELU, and
// either the store of X_{l+1} (feature d of the 42 nodes) or, in the last
// layer, the pooled sums the heads need.
template <typename OpT, int G_, bool LAST>
__device__ __forceinline__ void epilogue_graph(uint32_t tbase, float a_s, float a_n, float bias, float* s_self,
                                               float* s_nbr, float* inv_z, float* alpha, const int* rp_s,
                                               const uint32_t (&xs)[8], float& vs, float (&cs)[7], int lane) {
  float wh[kN];
#pragma unroll
  for (int t = 0; t < kN / 2; ++t) tmem_ld_x2(tbase + G_ * kN + 2 * t, wh[2 * t], wh[2 * t + 1]);
  tmem_ld_wait();
  // attention scores: reduce-scatter of a . Wh across the 32 feature lanes
  s_self[lane] = dot_scatter32<0>(wh, a_s, lane);
  s_nbr[lane] = dot_scatter32<0>(wh, a_n, lane);
  const float r3 = dot_scatter16<32>(wh, a_s, lane);
  const float r4 = dot_scatter16<32>(wh, a_n, lane);
  if (lane < 16) {
    s_self[32 + lane] = r3;
    s_nbr[32 + lane] = r4;
  }
  __syncwarp();
  // neighbour softmax over the 3x3 board stencil (the CSR in ascending
  // order); unnormalised weights in CSR order plus 1/z per node
  for (int i = lane; i < kN; i += 32) {
    const int r = i / 7, c = i % 7;
    const float si = s_self[i];
    float ev[9];
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < 9; ++k) {
      const int dr = k / 3 - 1, dc = k % 3 - 1;
      const bool in = (unsigned)(r + dr) < 6u && (unsigned)(c + dc) < 7u;
      ev[k] = in ? lrelu(si + s_nbr[i + 7 * dr + dc]) : -INFINITY;
      mx = fmaxf(mx, ev[k]);
    }
    int e = rp_s[i];
    float z = 0.f;
#pragma unroll
    for (int k = 0; k < 9; ++k) {
      if (ev[k] != -INFINITY) {
        const float pe = __expf(ev[k] - mx);
        alpha[e++] = pe;
        z += pe;
      }
    }
    inv_z[i] = 1.0f / z;
  }
  __syncwarp();
  const float4* a4 = (const float4*)alpha;
  const float4* z4 = (const float4*)inv_z;
  gather_rows<0>(wh, a4, [&](auto I, float acc) {
    constexpr int i = decltype(I)::value;
    const float x = elu_fast(fmaf(acc, pick4<i>(z4), bias));
    if constexpr (!LAST) {
      constexpr int j = G_ * kN + i;
      st_shared_u16<(j >> 3) * 1024 + (j & 7) * 128>(xs[j & 7], OpType<OpT>::bits(x));
    } else {
      vs += x;
      cs[i % 7] += x;
    }
  });
  __syncwarp();
}

struct TcParams {
  const uint8_t* packed;   // kChunksPerTile chunks in consumption order
  const float* w;          // fp32 blob (biases, attention vectors, heads)
  const int8_t* boards;
  const int8_t* side;
  float* pi;
  float* v;
  int* err;
  int n;
  int num_tiles;
};

template <typename OpT>
__global__ void __launch_bounds__(kThreads, 2) gat_tc_c4_kernel(TcParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  // The swizzled operand tiles need a 1024-byte aligned base.
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) atomicExch(p.err, 2);
    return;
  }
  uint8_t* sX = smem + kSmX;
  uint8_t* sW = smem + kSmW;
  float* scratch = (float*)(smem + kSmScratch);
  uint64_t* bars = (uint64_t*)(smem + kSmBar);
  uint64_t* full = bars;
  uint64_t* empty = bars + kSlots;
  uint64_t* acc_full = bars + 2 * kSlots;
  uint64_t* x_ready = acc_full + 1;
  uint64_t* drain = acc_full + 2;
  uint32_t* tmem_slot = (uint32_t*)(smem + kSmMisc);
  volatile int* abort_flag = (volatile int*)(smem + kSmMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  for (int i = threadIdx.x; i <= kN; i += blockDim.x) ((int*)(smem + kSmRp))[i] = c_rp[i];
  if (threadIdx.x == 0) {
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(x_ready, kEpiWarps);
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
          const int s = q % kSlots;
          ok = mbar_wait(&empty[s], ((q / kSlots) & 1) ^ 1, abort_flag, kWaitLimitNs);
          if (!ok) break;
          mbar_arrive_expect_tx(&full[s], kChunkBytes);
          bulk_g2s(sW + s * kChunkBytes, p.packed + (size_t)c * kChunkBytes, kChunkBytes, &full[s]);
        }
      }
      // Drain: every issued copy has landed before the CTA may exit.
      for (uint32_t k = (q > kSlots ? q - kSlots : 0); k < q; ++k)
        mbar_wait(&full[k % kSlots], (k / kSlots) & 1, abort_flag, kWaitLimitNs);
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(OpType<OpT>::fmt, 128, kTileCols);
      const uint32_t xs = smem_u32(sX);
      uint32_t q = 0, xphase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        for (int l = 0; l < kLayers && ok; ++l) {
          ok = mbar_wait(x_ready, xphase & 1, abort_flag, kWaitLimitNs);
          ++xphase;
          if (!ok) break;
          tc_fence_after();
          const int nchunk = l == 0 ? 1 : 4;   // K chunks of 64
          const int ksteps = l == 0 ? 1 : 4;   // K = 16 per MMA (layer 0: F = 4 -> one step)
          for (int m = 0; m < 2 && ok; ++m) {
            for (int c = 0; c < nchunk && ok; ++c, ++q) {
              const int s = q % kSlots;
              ok = mbar_wait(&full[s], (q / kSlots) & 1, abort_flag, kWaitLimitNs);
              if (!ok) break;
              tc_fence_after();
              const uint32_t ws = smem_u32(sW + s * kChunkBytes);
              for (int kk = 0; kk < ksteps; ++kk) {
                const uint64_t a = sw128_desc(ws + kk * 32);
                const uint64_t b = sw128_desc(xs + c * kChunkBytes + kk * 32);
                mma_f16_ss(tmem + m * kTileCols, a, b, idesc, (c | kk) != 0);
              }
              mma_commit(&empty[s]);
            }
          }
          if (ok) mma_commit(acc_full);
        }
      }
      mma_commit(drain);
      mbar_wait(drain, 0, abort_flag, kWaitLimitNs);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue: warp w owns head w ----------------
    const int h = warp;
    const int m = warp >> 2, qd = warp & 3;
    const int d = 128 * m + 32 * qd + lane;  // feature of this lane
    const uint32_t tbase = tmem + ((uint32_t)(32 * qd) << 16) + (uint32_t)(m * kTileCols);
    float* s_self = scratch + warp * kWarpScratchFloats;
    float* s_nbr = s_self + 48;
    float* inv_z = s_nbr + 48;
    float* alpha = inv_z + 48;
    const int* rp_s = (const int*)(smem + kSmRp);
    const int chunk_d = d >> 6, kk_d = d & 63;  // where feature d lives in the X tile
    // shared addresses of feature d in X-tile row r (mod 8) of the 128-byte
    // swizzle: row base + ((16-byte unit ^ r) << 4) + byte within the unit
    uint32_t xs[8];
#pragma unroll
    for (int r = 0; r < 8; ++r)
      xs[r] = smem_u32(sX + chunk_d * kChunkBytes) + ((((kk_d >> 3) ^ r) & 7) << 4) + (kk_d & 7) * 2;
    uint32_t aphase = 0;
    bool ok = true;

    for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
      // -- encode the tile's positions into X chunk 0 (features 0..15) --
      for (int t = threadIdx.x; t < kTileCols * 2; t += kEpiWarps * 32) {
        const int j = t >> 1, half = t & 1;
        const int g = j / kN, i = j % kN;
        const int pos = tile * kGPT + g;
        uint32_t wv[4] = {0, 0, 0, 0};
        if (half == 0 && g < kGPT && pos < p.n) {
          float f[4];
          encode_node(kConnect4, p.boards + (size_t)pos * 42, p.side[pos], i, f);
          wv[0] = (uint32_t)OpType<OpT>::bits(f[0]) | ((uint32_t)OpType<OpT>::bits(f[1]) << 16);
          wv[1] = (uint32_t)OpType<OpT>::bits(f[2]) | ((uint32_t)OpType<OpT>::bits(f[3]) << 16);
        }
        *(uint4*)(sX + sw128_offset(j, half * 8)) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(x_ready);

      for (int l = 0; l < kLayers && ok; ++l) {
        const float bias = __ldg(p.w + C4Off::b(l) + d);
        const float a_s = __ldg(p.w + C4Off::a(l) + (h * 2 + 0) * kHeadDim + lane);
        const float a_n = __ldg(p.w + C4Off::a(l) + (h * 2 + 1) * kHeadDim + lane);
        const bool last = l == kLayers - 1;
        ok = epilogue_all(mbar_wait(acc_full, aphase & 1, abort_flag, kWaitLimitNs));
        ++aphase;
        if (!ok) break;
        tc_fence_after();
        // head scratch lives in X chunks 1..3, unused from the last projection
        // until the next tile's first aggregation
        float* pooled = (float*)(sX + kChunkBytes);       // [3][256]
        float* pol = pooled + kGPT * 256;                 // [3][8 warps][8]
        float* zbuf = pol + kGPT * kEpiWarps * 8;         // [3][64]
        if (!last) {
          float vs = 0.f, cs[7];
          epilogue_graph<OpT, 0, false>(tbase, a_s, a_n, bias, s_self, s_nbr, inv_z, alpha, rp_s, xs, vs, cs, lane);
          epilogue_graph<OpT, 1, false>(tbase, a_s, a_n, bias, s_self, s_nbr, inv_z, alpha, rp_s, xs, vs, cs, lane);
          epilogue_graph<OpT, 2, false>(tbase, a_s, a_n, bias, s_self, s_nbr, inv_z, alpha, rp_s, xs, vs, cs, lane);
        } else {
          const float wpi = __ldg(p.w + C4Off::w_pi + d);
#pragma unroll 1
          for (int g = 0; g < kGPT; ++g) {
            float vs = 0.f, cs[7] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            if (g == 0) epilogue_graph<OpT, 0, true>(tbase, a_s, a_n, bias, s_self, s_nbr, inv_z, alpha, rp_s, xs, vs, cs, lane);
            if (g == 1) epilogue_graph<OpT, 1, true>(tbase, a_s, a_n, bias, s_self, s_nbr, inv_z, alpha, rp_s, xs, vs, cs, lane);
            if (g == 2) epilogue_graph<OpT, 2, true>(tbase, a_s, a_n, bias, s_self, s_nbr, inv_z, alpha, rp_s, xs, vs, cs, lane);
            pooled[g * 256 + d] = vs * (1.0f / kN);
#pragma unroll
            for (int c = 0; c < 7; ++c) {
              float t = cs[c] * (1.0f / 6.0f) * wpi;
#pragma unroll
              for (int o = 16; o >= 1; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
              if (lane == 0) pol[(g * kEpiWarps + warp) * 8 + c] = t;
            }
          }
        }
        tc_fence_before();
        if (!last) {
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(x_ready);
        } else {
          // ---------------- heads (fp32) ----------------
          named_bar_sync(1, kEpiWarps * 32);
          for (int t = threadIdx.x; t < kGPT * kValueHidden; t += kEpiWarps * 32) {
            const int g = t / kValueHidden, u = t % kValueHidden;
            float acc = __ldg(p.w + C4Off::b_v1 + u);
            for (int c = 0; c < 256; ++c)
              acc = fmaf(pooled[g * 256 + c], __ldg(p.w + C4Off::W_v1 + c * kValueHidden + u), acc);
            zbuf[g * kValueHidden + u] = fmaxf(acc, 0.f);
          }
          named_bar_sync(1, kEpiWarps * 32);
          if (warp < kGPT) {
            const int g = warp, pos = tile * kGPT + g;
            float vv = zbuf[g * kValueHidden + lane] * __ldg(p.w + C4Off::w_v2 + lane) +
                       zbuf[g * kValueHidden + 32 + lane] * __ldg(p.w + C4Off::w_v2 + 32 + lane);
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) vv += __shfl_xor_sync(0xffffffffu, vv, o);
            float lg = -INFINITY;
            if (lane < 7) {
              lg = __ldg(p.w + C4Off::b_pi);
              for (int w2 = 0; w2 < kEpiWarps; ++w2) lg += pol[(g * kEpiWarps + w2) * 8 + lane];
            }
            float mx = lg;
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            float ex = lane < 7 ? expf(lg - mx) : 0.f;
            float z = ex;
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
            if (pos < p.n) {
              if (lane < 7) p.pi[(size_t)pos * 7 + lane] = ex / z;
              if (lane == 0) p.v[pos] = tanhf(vv + __ldg(p.w + C4Off::b_v2));
            }
          }
          named_bar_sync(1, kEpiWarps * 32);  // scratch reused by the next tile
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

// ---- weight packing: W_l^T into swizzled 16 KB chunks ----
template <typename OpT>
__global__ void pack_c4_kernel(const float* __restrict__ w, uint8_t* __restrict__ out) {
  const GatLayout L = gat_layout(kConnect4);
  const int chunk = blockIdx.x;  // 0 .. kChunksPerTile-1
  int layer, m, c;
  if (chunk < 2) {
    layer = 0; m = chunk; c = 0;
  } else {
    layer = 1 + (chunk - 2) / 8;
    m = ((chunk - 2) % 8) / 4;
    c = (chunk - 2) % 4;
  }
  const int fin = layer == 0 ? 4 : 256;
  const float* W = w + L.W[layer];
  uint8_t* dst = out + (size_t)chunk * kChunkBytes;
  for (int t = threadIdx.x; t < 128 * 64; t += blockDim.x) {
    const int r = t / 64, kk = t % 64;
    const int k = c * 64 + kk, f = m * 128 + r;
    const float x = k < fin ? W[(size_t)k * kHidden + f] : 0.f;
    *(uint16_t*)(dst + sw128_offset(r, kk)) = OpType<OpT>::bits(x);
  }
}

int g_c4_graph_uploaded_dev = -1;

cudaError_t upload_c4_graph() {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  // constant memory is per device; upload unconditionally (cheap, idempotent)
  e = cudaMemcpyToSymbol(c_rp, kC4.rp, sizeof(kC4.rp));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(c_col, kC4.col, sizeof(kC4.col));
  if (e == cudaSuccess) g_c4_graph_uploaded_dev = dev;
  return e;
}

}  // namespace

size_t gat_tc_packed_bytes(int game) {
  return game == kConnect4 ? (size_t)kChunksPerTile * kChunkBytes : 0;
}

cudaError_t launch_gat_tc_pack(int game, int fp16, const float* d_weights, void* d_packed, cudaStream_t stream) {
  if (game != kConnect4) return cudaErrorNotSupported;
  cudaError_t e = upload_c4_graph();
  if (e != cudaSuccess) return e;
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
  // Per-device launch shape, computed once: persistent grid of
  // (SMs x resident CTAs per SM, at most two: tensor memory holds two CTAs'
  // 256-column accumulators).
  static int cached_grid[64][2];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  int& full_grid = cached_grid[dev][fp16 ? 1 : 0];
  if (full_grid == 0) {
    int sms = 0, per_sm = 0, smem_sm = 0, reserved = 0;
    if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemAlloc)) != cudaSuccess) return e;
    if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev)) != cudaSuccess) return e;
    if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, kSmemAlloc)) != cudaSuccess) return e;
    // The occupancy query can under-report here; shared memory (the binding
    // limit, registers are capped by __launch_bounds__) decides directly.
    const int by_smem = smem_sm / (kSmemAlloc + reserved);
    if (by_smem > per_sm) per_sm = by_smem;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    full_grid = sms * (per_sm > 2 ? 2 : per_sm);
  }
  int grid = full_grid;
  if (grid > p.num_tiles) grid = p.num_tiles;
  kern<<<grid, kThreads, kSmemAlloc, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace gz
