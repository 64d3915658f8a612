// Batched PUCT search kernels: one warp per tree.
//
// A wave selects `leaves` leaves per tree, one after another inside the
// owning warp, adding a virtual loss along each path so later selections of the
// same wave spread out; the leaves are evaluated as one network batch; the
// backup then expands first-visited leaves and propagates values in leaf
// order.  Because each tree is touched by exactly one warp and every step runs
// in a fixed order with explicitly rounded IEEE operations (no contraction),
// visit counts are bit-identical to a sequential CPU run of the same
// algorithm fed the same evaluations.
//
// Reference semantics (self_play/self_play.cu):
//   score    Q + c_puct * P * sqrt(N_parent) / (1 + n)           720-736
//   expand   children for the legal actions, P from the policy  698-718, 627-629
//   backup   N += 1, W += v, v = -v per level                    738-758
//   terminal value = -(outcome for the side to move)             611-613
// Additions the reference lacks: virtual loss (k virtual visits of value -1
// per selection in flight), legal-move renormalisation of P, Dirichlet noise
// at the root, lowest-action tie break.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "gz_games.h"
#include "gz_mcts.h"

namespace gz {
namespace {

constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ unsigned long long mix64(unsigned long long z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Counter-based random numbers: a pure function of (seed, a, b, c).
__device__ __forceinline__ unsigned long long rng64(unsigned long long seed, unsigned long long a, unsigned long long b,
                                                    unsigned long long c) {
  return mix64(seed ^ mix64(a ^ mix64(b ^ mix64(c))));
}
__device__ __forceinline__ float rng_unit(unsigned long long h) {  // (0, 1]
  return (float)((h >> 40) + 1) * (1.0f / 16777216.0f);
}

// Gamma(alpha, 1) by Marsaglia & Tsang (2000), with the alpha < 1 boost
// Gamma(alpha) = Gamma(alpha + 1) * U^(1/alpha).  Rejection is bounded.
__device__ float sample_gamma(float alpha, unsigned long long seed, unsigned long long a, unsigned long long b) {
  float boost = 1.0f;
  if (alpha < 1.0f) {
    boost = powf(rng_unit(rng64(seed, a, b, 0xB0)), 1.0f / alpha);
    alpha += 1.0f;
  }
  const float dd = alpha - 1.0f / 3.0f, cc = rsqrtf(9.0f * dd);
  for (int it = 0; it < 64; ++it) {
    float u1 = rng_unit(rng64(seed, a, b, 4 * it + 1));
    float u2 = rng_unit(rng64(seed, a, b, 4 * it + 2));
    float x = sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);  // Box-Muller
    float t = 1.0f + cc * x;
    if (t <= 0.0f) continue;
    float vv = t * t * t;
    float u = rng_unit(rng64(seed, a, b, 4 * it + 3));
    if (logf(u) < 0.5f * x * x + dd - dd * vv + dd * logf(vv)) return dd * vv * boost;
  }
  return dd * boost;
}

__device__ __forceinline__ void set_err(int* err, int code) { atomicCAS(err, 0, code); }

__device__ void init_node(const MctsDev& d, size_t gnode, const int8_t* board, int side, int terminal, float tv) {
  d.n[gnode] = 0;
  d.vl[gnode] = 0;
  d.first_edge[gnode] = -1;
  d.n_edges[gnode] = 0;
  d.side[gnode] = (int8_t)side;
  d.expanded[gnode] = 0;
  d.terminal[gnode] = (int8_t)terminal;
  d.term_value[gnode] = tv;
  int8_t* dst = d.board + gnode * kMctsBoardStride;
  for (int i = 0; i < kMctsBoardStride; ++i) dst[i] = i < d.N ? board[i] : 0;
}

__global__ void reset_kernel(MctsDev d, const int8_t* __restrict__ boards, const int8_t* __restrict__ side) {
  int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= d.trees) return;
  d.root[t] = 0;
  d.node_count[t] = 1;
  d.edge_count[t] = 0;
  d.move_no[t] = 0;
  init_node(d, (size_t)t * d.node_cap, boards + (size_t)t * d.N, side[t], 0, 0.0f);
}

__global__ void select_kernel(MctsDev d) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= d.trees) return;
  const size_t nb = (size_t)t * d.node_cap, eb = (size_t)t * d.edge_cap;
  for (int k = 0; k < d.leaves; ++k) {
    const size_t slot = (size_t)t * d.leaves + k;
    int* pn = d.path_nodes + slot * kMctsMaxDepth;
    int* pe = d.path_edges + slot * kMctsMaxDepth;
    int s = d.root[t];
    int depth = 0;
    if (lane == 0) pn[0] = s;
    while (true) {
      // the node's fields in one round of loads (read before the test: the
      // fields of an unexpanded node are read and not used)
      const size_t gs = nb + s;
      const int8_t expanded = d.expanded[gs], terminal = d.terminal[gs];
      const int ne = d.n_edges[gs], fe = d.first_edge[gs];
      const int vl_s = d.vl[gs];
      const int np = d.n[gs] + d.vl_k * vl_s;
      if (!expanded || terminal) break;
      const float sq = __fsqrt_rn((float)np);
      float u = -INFINITY;
      int idx = 0x7fffffff;
      int child = -1;  // this lane's edge's child and virtual visits, loaded with its statistics
      int vl_e = 0;
      if (lane < ne) {
        const size_t e = eb + fe + lane;
        child = d.child[e];
        vl_e = d.VL[e];
        const int vlk = d.vl_k * vl_e;
        const int nev = d.Nv[e] + vlk;
        const float q = nev > 0 ? __fdiv_rn(__fsub_rn(d.W[e], (float)vlk), (float)nev) : 0.0f;
        const float u1 = __fmul_rn(d.c_puct, d.P[e]);
        const float u2 = __fmul_rn(u1, sq);
        const float u3 = __fdiv_rn(u2, __fadd_rn(1.0f, (float)nev));
        u = __fadd_rn(q, u3);
        idx = lane;
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        const float uo = __shfl_xor_sync(kFull, u, o);
        const int io = __shfl_xor_sync(kFull, idx, o);
        if (uo > u || (uo == u && io < idx)) { u = uo; idx = io; }
      }
      const int e = fe + idx;
      int c = __shfl_sync(kFull, child, idx);
      const int vl_c = __shfl_sync(kFull, vl_e, idx);
      if (lane == 0) {  // virtual visits: the values loaded above, stored back incremented
        d.vl[nb + s] = vl_s + 1;
        d.VL[eb + e] = vl_c + 1;
        if (c < 0) {
          c = d.node_count[t];
          if (c >= d.node_cap) {
            set_err(d.err, kMctsNodeCap);
            c = -1;
          } else {
            d.node_count[t] = c + 1;
            int8_t b[kMctsBoardStride];
            const int8_t* pb = d.board + (nb + s) * kMctsBoardStride;
            for (int i = 0; i < kMctsBoardStride; ++i) b[i] = pb[i];
            const int mover = d.side[nb + s];
            const int sq_written = apply_action(d.game, b, d.action[eb + e], mover);
            const int oc = outcome_after(d.game, b, sq_written, mover);
            init_node(d, nb + c, b, -mover, oc != 0, oc == 1 ? -1.0f : 0.0f);
            d.child[eb + e] = c;
          }
        }
        if (depth + 1 >= kMctsMaxDepth) {
          set_err(d.err, kMctsDepth);
          c = -1;
        }
        if (c >= 0) {
          pe[depth] = e;
          pn[depth + 1] = c;
        }
      }
      c = __shfl_sync(kFull, c, 0);
      __syncwarp();
      if (c < 0) break;
      ++depth;
      s = c;
    }
    if (lane == 0) {
      d.vl[nb + s] += 1;
      d.path_len[slot] = depth;
      d.leaf_side[slot] = d.side[nb + s];
      d.leaf_terminal[slot] = d.terminal[nb + s];
    }
    for (int i = lane; i < d.N; i += 32) d.leaf_board[slot * d.N + i] = d.board[(nb + s) * kMctsBoardStride + i];
    __syncwarp();
  }
}

__global__ void backup_kernel(MctsDev d, const float* __restrict__ pi, const float* __restrict__ value) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= d.trees) return;
  const size_t nb = (size_t)t * d.node_cap, eb = (size_t)t * d.edge_cap;
  for (int k = 0; k < d.leaves; ++k) {
    const size_t slot = (size_t)t * d.leaves + k;
    const int* pn = d.path_nodes + slot * kMctsMaxDepth;
    const int* pe = d.path_edges + slot * kMctsMaxDepth;
    const int len = d.path_len[slot];
    const int leaf = pn[len];
    const size_t gl = nb + leaf;
    float val;
    if (d.terminal[gl]) {
      val = d.term_value[gl];
    } else {
      val = value[slot];
      if (!d.expanded[gl]) {
        const int8_t* bd = d.board + gl * kMctsBoardStride;
        const float* p = pi + slot * d.A;
        const bool lg = lane < d.A && action_legal(d.game, bd, lane);
        const unsigned mask = __ballot_sync(kFull, lg);
        const int cnt = __popc(mask);
        float sum = 0.0f;
        int fe = 0;
        if (lane == 0) {
          for (int a = 0; a < d.A; ++a)
            if ((mask >> a) & 1u) sum = __fadd_rn(sum, p[a]);
          fe = d.edge_count[t];
          if (fe + cnt > d.edge_cap) {
            set_err(d.err, kMctsEdgeCap);
            fe = -1;
          } else {
            d.edge_count[t] = fe + cnt;
          }
        }
        sum = __shfl_sync(kFull, sum, 0);
        fe = __shfl_sync(kFull, fe, 0);
        if (fe >= 0) {
          if (lg) {
            const size_t e = eb + fe + __popc(mask & ((1u << lane) - 1u));
            d.P[e] = __fdiv_rn(p[lane], sum);
            d.W[e] = 0.0f;
            d.Nv[e] = 0;
            d.VL[e] = 0;
            d.child[e] = -1;
            d.action[e] = (int8_t)lane;
          }
          __syncwarp();
          if (lane == 0) {
            if (d.dir_eps > 0.0f && leaf == d.root[t] && cnt > 0) {
              // Root exploration noise: P = (1 - eps) P + eps Dir(alpha).
              float g[32], gs = 0.0f;
              for (int j = 0; j < cnt; ++j) {
                g[j] = sample_gamma(d.dir_alpha, d.seed, (unsigned long long)t, ((unsigned long long)d.move_no[t] << 8) | j);
                gs += g[j];
              }
              for (int j = 0; j < cnt; ++j) {
                const size_t e = eb + fe + j;
                d.P[e] = (1.0f - d.dir_eps) * d.P[e] + d.dir_eps * (gs > 0.0f ? g[j] / gs : 1.0f / cnt);
              }
            }
            d.first_edge[gl] = fe;
            d.n_edges[gl] = (int8_t)cnt;
            d.expanded[gl] = 1;
          }
        }
      }
    }
    __syncwarp();
    // The path's levels touch distinct nodes and edges, so the lanes update
    // them at once; the value at level i is -val for i = len - 1 and changes
    // sign every level up (the same additions as a walk from the leaf, and
    // the leaves of a tree still back up in order).
    if (lane == 0) {
      d.n[gl] += 1;
      d.vl[gl] -= 1;
    }
    for (int i = lane; i < len; i += 32) {
      const float x = ((len - 1 - i) & 1) ? val : -val;
      const size_t e = eb + pe[i];
      d.Nv[e] += 1;
      d.W[e] = __fadd_rn(d.W[e], x);
      d.VL[e] -= 1;
      const size_t gs = nb + pn[i];
      d.n[gs] += 1;
      d.vl[gs] -= 1;
    }
    __syncwarp();
  }
}

__global__ void root_visits_kernel(MctsDev d, int32_t* __restrict__ visits, float* __restrict__ wsum) {
  int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= d.trees) return;
  const size_t nb = (size_t)t * d.node_cap, eb = (size_t)t * d.edge_cap;
  for (int a = 0; a < d.A; ++a) {
    visits[(size_t)t * d.A + a] = 0;
    if (wsum) wsum[(size_t)t * d.A + a] = 0.0f;
  }
  const int r = d.root[t];
  if (!d.expanded[nb + r]) return;
  const int fe = d.first_edge[nb + r], ne = d.n_edges[nb + r];
  for (int k = 0; k < ne; ++k) {
    const size_t e = eb + fe + k;
    visits[(size_t)t * d.A + d.action[e]] = d.Nv[e];
    if (wsum) wsum[(size_t)t * d.A + d.action[e]] = d.W[e];
  }
}

// Move choice (reference: mcts_get_policy N^(1/T), self_play.cu:645-662, and
// CDF sampling, 675-686): T = 1 for the first temp_moves moves of a game,
// sampling an action with probability N_a / sum N; afterwards the most visited
// action (lowest action on ties).  Integer arithmetic only.
__global__ void choose_kernel(MctsDev d, int temp_moves, int32_t* __restrict__ actions) {
  int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= d.trees) return;
  const size_t nb = (size_t)t * d.node_cap, eb = (size_t)t * d.edge_cap;
  const int r = d.root[t];
  const int fe = d.first_edge[nb + r], ne = d.expanded[nb + r] ? (int)d.n_edges[nb + r] : 0;
  int pick = -1;
  if (ne > 0) {
    long long total = 0;
    int best = 0;
    for (int k = 0; k < ne; ++k) {
      int nv = d.Nv[eb + fe + k];
      total += nv;
      if (nv > d.Nv[eb + fe + best]) best = k;
    }
    pick = best;
    if (d.move_no[t] < temp_moves && total > 0) {
      unsigned long long h = rng64(d.seed, (unsigned long long)t, (unsigned long long)d.move_no[t], 0xC4);
      long long x = (long long)(((h >> 32) * (unsigned long long)total) >> 32);
      long long cum = 0;
      for (int k = 0; k < ne; ++k) {
        cum += d.Nv[eb + fe + k];
        if (cum > x) { pick = k; break; }
      }
    }
  }
  if (pick >= 0) {
    actions[t] = d.action[eb + fe + pick];
  } else {  // unexpanded root: first legal action
    const int8_t* bd = d.board + (nb + r) * kMctsBoardStride;
    int a = 0;
    while (a < d.A - 1 && !action_legal(d.game, bd, a)) ++a;
    actions[t] = a;
  }
}

// Advance roots (reference mcts_update_with_move, mcts/mcts.cu:68-103): the
// child keeps its subtree while `reserve` nodes remain free in the pool;
// otherwise the pool restarts from the new position.  A finished game
// restarts from the empty board with the first player to move.
__global__ void play_kernel(MctsDev d, const int32_t* __restrict__ actions, int reserve, int8_t* __restrict__ done) {
  int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= d.trees) return;
  const size_t nb = (size_t)t * d.node_cap, eb = (size_t)t * d.edge_cap;
  const int r = d.root[t];
  const int a = actions[t];
  int child = -1;
  if (d.expanded[nb + r]) {
    const int fe = d.first_edge[nb + r], ne = d.n_edges[nb + r];
    for (int k = 0; k < ne; ++k)
      if (d.action[eb + fe + k] == a) child = d.child[eb + fe + k];
  }
  int8_t b[kMctsBoardStride];
  for (int i = 0; i < kMctsBoardStride; ++i) b[i] = d.board[(nb + r) * kMctsBoardStride + i];
  const int mover = d.side[nb + r];
  const int sq = apply_action(d.game, b, a, mover);
  const int oc = sq < 0 ? 2 : outcome_after(d.game, b, sq, mover);
  if (done) done[t] = (int8_t)(oc != 0);
  if (oc != 0) {
    for (int i = 0; i < kMctsBoardStride; ++i) b[i] = 0;
    d.root[t] = 0;
    d.node_count[t] = 1;
    d.edge_count[t] = 0;
    d.move_no[t] = 0;
    init_node(d, nb, b, 1, 0, 0.0f);
  } else if (child >= 0 && d.node_count[t] + reserve <= d.node_cap) {
    d.root[t] = child;
    d.move_no[t] += 1;
  } else {
    d.root[t] = 0;
    d.node_count[t] = 1;
    d.edge_count[t] = 0;
    d.move_no[t] += 1;
    init_node(d, nb, b, -mover, 0, 0.0f);
  }
}

__global__ void tree_sizes_kernel(MctsDev d, int32_t* nodes, int32_t* edges) {
  int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= d.trees) return;
  nodes[t] = d.node_count[t];
  edges[t] = d.edge_count[t];
}

inline int blocks_for(int n, int per) { return (n + per - 1) / per; }

}  // namespace

cudaError_t mcts_launch_reset(const MctsDev& d, const int8_t* boards, const int8_t* side, cudaStream_t s) {
  reset_kernel<<<blocks_for(d.trees, 128), 128, 0, s>>>(d, boards, side);
  return cudaGetLastError();
}

cudaError_t mcts_launch_select(const MctsDev& d, cudaStream_t s) {
  select_kernel<<<blocks_for(d.trees, 4), 128, 0, s>>>(d);
  return cudaGetLastError();
}

cudaError_t mcts_launch_backup(const MctsDev& d, const float* pi, const float* v, cudaStream_t s) {
  backup_kernel<<<blocks_for(d.trees, 4), 128, 0, s>>>(d, pi, v);
  return cudaGetLastError();
}

cudaError_t mcts_launch_root_visits(const MctsDev& d, int32_t* visits, float* wsum, cudaStream_t s) {
  root_visits_kernel<<<blocks_for(d.trees, 128), 128, 0, s>>>(d, visits, wsum);
  return cudaGetLastError();
}

cudaError_t mcts_launch_choose(const MctsDev& d, int temp_moves, int32_t* actions, cudaStream_t s) {
  choose_kernel<<<blocks_for(d.trees, 128), 128, 0, s>>>(d, temp_moves, actions);
  return cudaGetLastError();
}

cudaError_t mcts_launch_play(const MctsDev& d, const int32_t* actions, int reserve, int8_t* done, cudaStream_t s) {
  play_kernel<<<blocks_for(d.trees, 128), 128, 0, s>>>(d, actions, reserve, done);
  return cudaGetLastError();
}

cudaError_t mcts_launch_tree_sizes(const MctsDev& d, int32_t* nodes, int32_t* edges, cudaStream_t s) {
  tree_sizes_kernel<<<blocks_for(d.trees, 128), 128, 0, s>>>(d, nodes, edges);
  return cudaGetLastError();
}

}  // namespace gz
