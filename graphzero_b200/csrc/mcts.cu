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
// Memory: a tree is one contiguous pool of 32-byte edge records (gz_mcts.h).
// A selection level loads the current node's edges (one record per lane, one
// round of loads) and nothing else: the chosen edge already carries the
// child's counts, flags and first edge.  The position is carried down the
// path in registers, two cells per lane, and the rules run warp-wide on it
// (ballots over the cells), so creating a leaf reads no stored position.
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

#include "gz_chess.h"
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

__device__ __forceinline__ uint32_t make_meta(uint32_t action, int n_edges, uint32_t flags) {
  return action | ((uint32_t)n_edges << 8) | (flags << 16);
}

// ---------------------------------------------------------------------------
// Warp-wide rules on a position held two cells per lane: lane j holds cell j
// (`lo`) and cell 32 + j (`hi`), 0 where the board has no such cell.  They
// restate gz_games.h's apply_action / outcome_after / action_legal with
// ballots; every lane must call them.
// ---------------------------------------------------------------------------

// Apply action a for player p; returns the square written or -1 (apply_action).
__device__ __forceinline__ int warp_apply(int game, int N, int& lo, int& hi, int a, int p, int lane) {
  if (game == kConnect4) {
    // the lowest empty cell of column a: the empty cell r * 7 + a with the largest r
    const unsigned mlo = __ballot_sync(kFull, lane < N && lane % 7 == a && lo == 0);
    const unsigned mhi = __ballot_sync(kFull, lane + 32 < N && (lane + 32) % 7 == a && hi == 0);
    const int sq = mhi ? 63 - __clz(mhi) : (mlo ? 31 - __clz(mlo) : -1);
    if (sq == lane) lo = p;
    if (sq == lane + 32) hi = p;
    return sq;
  }
  const int cell = __shfl_sync(kFull, lo, a & 31);
  if (a < 0 || a >= N || cell != 0) return -1;
  if (lane == a) lo = p;
  return a;
}

// Outcome after player p wrote `sq`: 1 = p won, 2 = draw (board full), 0 = the
// game continues (outcome_after: Connect4 counts the lines through sq,
// TicTacToe tests all eight lines).
__device__ __forceinline__ int warp_outcome(int game, int N, int lo, int hi, int sq, int p, int lane) {
  const unsigned long long mine =
      (unsigned long long)__ballot_sync(kFull, lane < N && lo == p) |
      ((unsigned long long)__ballot_sync(kFull, lane + 32 < N && hi == p) << 32);
  const unsigned filled = __ballot_sync(kFull, lane < N && lo != 0);
  bool win = false;
  if (game == kConnect4) {
    // lane j < 16: the window of four in direction j / 4 that holds sq at
    // position j % 4
    if (lane < 16 && sq >= 0) {
      const int dir = lane >> 2, off = lane & 3;
      const int dr = dir == 0 ? 0 : 1, dc = dir == 0 ? 1 : (dir == 1 ? 0 : (dir == 2 ? 1 : -1));
      const int r0 = sq / 7 - off * dr, c0 = sq % 7 - off * dc;
      win = true;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int r = r0 + k * dr, c = c0 + k * dc;
        win = win && r >= 0 && r < 6 && c >= 0 && c < 7 && ((mine >> (r * 7 + c)) & 1ull);
      }
    }
  } else if (lane < 8) {
    // rows (lanes 0-2), columns (3-5), diagonals (6, 7)
    const int a = lane < 3 ? 3 * lane : (lane < 6 ? lane - 3 : (lane == 6 ? 0 : 2));
    const int st = lane < 3 ? 1 : (lane < 6 ? 3 : (lane == 6 ? 4 : 2));
    win = ((mine >> a) & 1ull) && ((mine >> (a + st)) & 1ull) && ((mine >> (a + 2 * st)) & 1ull);
  }
  if (__any_sync(kFull, win)) return 1;
  const unsigned need = game == kConnect4 ? 0x7fu : 0x1ffu;  // Connect4: full iff the top row is
  return (filled & need) == need ? 2 : 0;
}

// Legal actions (action_legal): cell a empty, a < A (the top row for Connect4).
__device__ __forceinline__ uint32_t warp_legal(int A, int lo, int lane) {
  return __ballot_sync(kFull, lane < A && lo == 0);
}

__device__ void reset_tree(MctsTree* tr, const int8_t* board, int N, int side, int move_no) {
  for (int i = 0; i < kMctsBoardStride; ++i) tr->board[i] = i < N ? board[i] : (int8_t)0;
  tr->fe = -1;
  tr->meta = make_meta(0, 0, kNodeCreated);
  tr->n = 0;
  tr->vl = 0;
  tr->node_count = 1;
  tr->edge_count = 0;
  tr->move_no = move_no;
  tr->side = side;
}

__global__ void reset_kernel(MctsDev d, const int8_t* __restrict__ boards, const int8_t* __restrict__ side) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= d.trees) return;
  reset_tree(d.tree + t, boards + (size_t)t * d.N, d.N, side[t], 0);
}

// One wave's selections on tree t (all 32 lanes of a warp).
__device__ __forceinline__ void select_tree(const MctsDev& d, int t, int lane) {
  MctsTree* tr = d.tree + t;
  MctsEdge* E = d.edges + (size_t)t * d.edge_cap;
  const int N = d.N;
  // the root's record: one 128-byte line
  const int r_fe = tr->fe;
  const uint32_t r_meta = tr->meta;
  const int r_n = tr->n, r_side = tr->side;
  int r_vl = tr->vl;
  int node_count = tr->node_count;
  const int r_lo = lane < N ? tr->board[lane] : 0;
  const int r_hi = lane + 32 < N ? tr->board[lane + 32] : 0;
  for (int k = 0; k < d.leaves; ++k) {
    const size_t slot = (size_t)t * d.leaves + k;
    int* pe = d.path_edges + slot * kMctsMaxDepth;
    int fe = r_fe, ne = meta_edges(r_meta);
    uint32_t flags = meta_flags(r_meta);
    int np = r_n + d.vl_k * r_vl;  // N_parent with the virtual visits in flight
    r_vl += 1;
    int lo = r_lo, hi = r_hi, side = r_side, depth = 0;
    while ((flags & kNodeExpanded) && !(flags & kNodeTerminal)) {
      const float sq = __fsqrt_rn((float)np);
      float u = -INFINITY;
      int idx = 0x7fffffff;
      int4 ra = make_int4(0, 0, 0, 0), rb = make_int4(0, 0, 0, 0);
      if (lane < ne) {  // this lane's edge: P, W, Nv, VL | child_fe, meta
        const int4* rec = (const int4*)(E + fe + lane);
        ra = rec[0];
        rb = rec[1];
        const int vlk = d.vl_k * ra.w;
        const int nev = ra.z + vlk;
        const float q = nev > 0 ? __fdiv_rn(__fsub_rn(__int_as_float(ra.y), (float)vlk), (float)nev) : 0.0f;
        const float u1 = __fmul_rn(d.c_puct, __int_as_float(ra.x));
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
      const int c_nv = __shfl_sync(kFull, ra.z, idx), c_vl = __shfl_sync(kFull, ra.w, idx);
      const int c_fe = __shfl_sync(kFull, rb.x, idx);
      const uint32_t c_meta = (uint32_t)__shfl_sync(kFull, rb.y, idx);
      uint32_t cflags = meta_flags(c_meta);
      if (!(cflags & kNodeCreated) && node_count >= d.node_cap) {
        if (lane == 0) set_err(d.err, kMctsNodeCap);
        break;
      }
      if (depth + 1 >= kMctsMaxDepth) {
        if (lane == 0) set_err(d.err, kMctsDepth);
        break;
      }
      if (lane == 0) {  // a virtual visit on the edge (and so on the child); the path
        E[e].VL = c_vl + 1;
        pe[depth] = e;
      }
      const int mover = side;
      const int sqw = warp_apply(d.game, N, lo, hi, (int)meta_action(c_meta), mover, lane);
      side = -side;
      ++depth;
      if (!(cflags & kNodeCreated)) {  // a new node: counted, and the game may end there
        ++node_count;
        const int oc = warp_outcome(d.game, N, lo, hi, sqw, mover, lane);
        cflags = kNodeCreated | (oc != 0 ? kNodeTerminal : 0u) | (oc == 1 ? kNodeLoss : 0u);
        if (lane == 0) E[e].meta = make_meta(meta_action(c_meta), 0, cflags);
      }
      flags = cflags;
      fe = c_fe;
      ne = meta_edges(c_meta);
      np = c_nv + d.vl_k * c_vl;
    }
    const uint32_t legal = warp_legal(d.A, lo, lane);
    if (lane == 0) {
      d.path_len[slot] = depth;
      d.leaf_side[slot] = (int8_t)side;
      d.leaf_terminal[slot] = (flags & kNodeTerminal) ? 1 : 0;
      d.leaf_legal[slot] = legal;
    }
    int8_t* lb = d.leaf_board + slot * N;
    if (lane < N) lb[lane] = (int8_t)lo;
    if (lane + 32 < N) lb[lane + 32] = (int8_t)hi;
  }
  if (lane == 0) {
    tr->vl = r_vl;
    tr->node_count = node_count;
  }
}

// Expansion and backup of the wave's leaves of tree t (all 32 lanes of a warp).
__device__ __forceinline__ void backup_tree(const MctsDev& d, const float* __restrict__ pi,
                                            const float* __restrict__ value, int t, int lane) {
  MctsTree* tr = d.tree + t;
  MctsEdge* E = d.edges + (size_t)t * d.edge_cap;
  int r_fe = tr->fe;
  uint32_t r_meta = tr->meta;
  int r_n = tr->n, r_vl = tr->vl, edge_count = tr->edge_count;
  const int move_no = tr->move_no;
  for (int k = 0; k < d.leaves; ++k) {
    const size_t slot = (size_t)t * d.leaves + k;
    const int* pe = d.path_edges + slot * kMctsMaxDepth;
    const int len = d.path_len[slot];
    // the path's edges, level i in lane i % 32
    const int e0 = lane < len ? pe[lane] : -1;
    const int e1 = lane + 32 < len ? pe[lane + 32] : -1;
    const int le = len > 0 ? __shfl_sync(kFull, len - 1 < 32 ? e0 : e1, (len - 1) & 31) : -1;  // edge into the leaf
    uint32_t lmeta = r_meta;
    if (len > 0 && lane == 0) lmeta = E[le].meta;  // read and written by lane 0 only
    lmeta = __shfl_sync(kFull, lmeta, 0);
    const uint32_t lflags = meta_flags(lmeta);
    float val;
    if (lflags & kNodeTerminal) {
      val = (lflags & kNodeLoss) ? -1.0f : 0.0f;
    } else {
      val = value[slot];
      if (!(lflags & kNodeExpanded)) {
        const float* p = pi + slot * d.A;
        const bool lg = lane < d.A && ((d.leaf_legal[slot] >> lane) & 1u);
        const unsigned mask = __ballot_sync(kFull, lg);
        const int cnt = __popc(mask);
        float sum = 0.0f;
        int fe = 0;
        if (lane == 0) {
          for (int a = 0; a < d.A; ++a)
            if ((mask >> a) & 1u) sum = __fadd_rn(sum, p[a]);
          fe = edge_count;
          if (fe + cnt > d.edge_cap) {
            set_err(d.err, kMctsEdgeCap);
            fe = -1;
          } else {
            edge_count = fe + cnt;
          }
        }
        sum = __shfl_sync(kFull, sum, 0);
        fe = __shfl_sync(kFull, fe, 0);
        if (fe >= 0) {
          if (lg) {
            int4* rec = (int4*)(E + fe + __popc(mask & ((1u << lane) - 1u)));
            rec[0] = make_int4(__float_as_int(__fdiv_rn(p[lane], sum)), __float_as_int(0.0f), 0, 0);
            rec[1] = make_int4(-1, (int)make_meta((uint32_t)lane, 0, 0), 0, 0);
          }
          __syncwarp();
          if (lane == 0) {
            if (d.dir_eps > 0.0f && len == 0 && cnt > 0) {
              // Root exploration noise: P = (1 - eps) P + eps Dir(alpha).
              float g[32], gs = 0.0f;
              for (int j = 0; j < cnt; ++j) {
                g[j] = sample_gamma(d.dir_alpha, d.seed, (unsigned long long)t, ((unsigned long long)move_no << 8) | j);
                gs += g[j];
              }
              for (int j = 0; j < cnt; ++j)
                E[fe + j].P = (1.0f - d.dir_eps) * E[fe + j].P + d.dir_eps * (gs > 0.0f ? g[j] / gs : 1.0f / cnt);
            }
            const uint32_t nm = make_meta(meta_action(lmeta), cnt, lflags | kNodeExpanded);
            if (len > 0) {
              E[le].child_fe = fe;
              E[le].meta = nm;
            } else {
              r_fe = fe;
              r_meta = nm;
            }
          }
          r_fe = __shfl_sync(kFull, r_fe, 0);
          r_meta = __shfl_sync(kFull, r_meta, 0);
        }
      }
    }
    __syncwarp();
    // Every level's edge gets the visit, the value and its virtual visit
    // back; the levels are distinct edges, so the lanes update them at once.
    // The value at level i is -val for i = len - 1 and changes sign every
    // level up (the same additions as a walk from the leaf; the leaves of a
    // tree still back up in order, and level i is always lane i % 32).
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int i = lane + 32 * h, e = h ? e1 : e0;
      if (i < len) {
        const float x = ((len - 1 - i) & 1) ? val : -val;
        int4* rec = (int4*)(E + e);
        int4 s = rec[0];
        s.y = __float_as_int(__fadd_rn(__int_as_float(s.y), x));
        s.z += 1;
        s.w -= 1;
        rec[0] = s;
      }
    }
    r_n += 1;
    r_vl -= 1;
    __syncwarp();
  }
  if (lane == 0) {
    tr->fe = r_fe;
    tr->meta = r_meta;
    tr->n = r_n;
    tr->vl = r_vl;
    tr->edge_count = edge_count;
  }
}

__global__ void select_kernel(MctsDev d) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (t < d.trees) select_tree(d, t, threadIdx.x & 31);
}

__global__ void backup_kernel(MctsDev d, const float* __restrict__ pi, const float* __restrict__ value) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (t < d.trees) backup_tree(d, pi, value, t, threadIdx.x & 31);
}

// A wave's backup followed by the next wave's selections in the same warp:
// one launch instead of two between network passes (the warp's own writes
// are visible to its lanes after the barrier).
__global__ void backup_select_kernel(MctsDev d, const float* __restrict__ pi, const float* __restrict__ value) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (t >= d.trees) return;
  backup_tree(d, pi, value, t, threadIdx.x & 31);
  __syncwarp();
  select_tree(d, t, threadIdx.x & 31);
}

__global__ void root_visits_kernel(MctsDev d, int32_t* __restrict__ visits, float* __restrict__ wsum) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= d.trees) return;
  const MctsTree* tr = d.tree + t;
  const MctsEdge* E = d.edges + (size_t)t * d.edge_cap;
  for (int a = 0; a < d.A; ++a) {
    visits[(size_t)t * d.A + a] = 0;
    if (wsum) wsum[(size_t)t * d.A + a] = 0.0f;
  }
  if (!(meta_flags(tr->meta) & kNodeExpanded)) return;
  const int fe = tr->fe, ne = meta_edges(tr->meta);
  for (int k = 0; k < ne; ++k) {
    const MctsEdge& e = E[fe + k];
    visits[(size_t)t * d.A + meta_action(e.meta)] = e.Nv;
    if (wsum) wsum[(size_t)t * d.A + meta_action(e.meta)] = e.W;
  }
}

// Move choice (reference: mcts_get_policy N^(1/T), self_play.cu:645-662, and
// CDF sampling, 675-686): T = 1 for the first temp_moves moves of a game,
// sampling an action with probability N_a / sum N; afterwards the most visited
// action (lowest action on ties).  Integer arithmetic only.
__global__ void choose_kernel(MctsDev d, int temp_moves, int32_t* __restrict__ actions) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= d.trees) return;
  const MctsTree* tr = d.tree + t;
  const MctsEdge* E = d.edges + (size_t)t * d.edge_cap;
  const int fe = tr->fe, ne = (meta_flags(tr->meta) & kNodeExpanded) ? meta_edges(tr->meta) : 0;
  int pick = -1;
  if (ne > 0) {
    long long total = 0;
    int best = 0;
    for (int k = 0; k < ne; ++k) {
      const int nv = E[fe + k].Nv;
      total += nv;
      if (nv > E[fe + best].Nv) best = k;
    }
    pick = best;
    if (tr->move_no < temp_moves && total > 0) {
      const unsigned long long h = rng64(d.seed, (unsigned long long)t, (unsigned long long)tr->move_no, 0xC4);
      const long long x = (long long)(((h >> 32) * (unsigned long long)total) >> 32);
      long long cum = 0;
      for (int k = 0; k < ne; ++k) {
        cum += E[fe + k].Nv;
        if (cum > x) { pick = k; break; }
      }
    }
  }
  if (pick >= 0) {
    actions[t] = (int32_t)meta_action(E[fe + pick].meta);
  } else {  // unexpanded root: first legal action
    int a = 0;
    while (a < d.A - 1 && !action_legal(d.game, tr->board, a)) ++a;
    actions[t] = a;
  }
}

// Advance roots (reference mcts_update_with_move, mcts/mcts.cu:68-103): the
// child keeps its subtree while `reserve` nodes remain free in the pool;
// otherwise the pool restarts from the new position.  A finished game
// restarts from the empty board with the first player to move.
__global__ void play_kernel(MctsDev d, const int32_t* __restrict__ actions, int reserve, int8_t* __restrict__ done) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= d.trees) return;
  MctsTree* tr = d.tree + t;
  const MctsEdge* E = d.edges + (size_t)t * d.edge_cap;
  const int a = actions[t];
  const MctsEdge* ce = nullptr;  // the edge of the played action, if its child exists
  if (meta_flags(tr->meta) & kNodeExpanded) {
    const int fe = tr->fe, ne = meta_edges(tr->meta);
    for (int k = 0; k < ne; ++k)
      if ((int)meta_action(E[fe + k].meta) == a && (meta_flags(E[fe + k].meta) & kNodeCreated)) ce = E + fe + k;
  }
  int8_t b[kMctsBoardStride];
  for (int i = 0; i < kMctsBoardStride; ++i) b[i] = tr->board[i];
  const int mover = tr->side;
  const int sq = apply_action(d.game, b, a, mover);
  const int oc = sq < 0 ? 2 : outcome_after(d.game, b, sq, mover);
  if (done) done[t] = (int8_t)(oc != 0);
  if (oc != 0) {
    for (int i = 0; i < kMctsBoardStride; ++i) b[i] = 0;
    reset_tree(tr, b, d.N, 1, 0);
  } else if (ce && tr->node_count + reserve <= d.node_cap) {
    for (int i = 0; i < kMctsBoardStride; ++i) tr->board[i] = b[i];
    tr->fe = ce->child_fe;
    tr->meta = make_meta(0, meta_edges(ce->meta), meta_flags(ce->meta));
    tr->n = ce->Nv;
    tr->vl = ce->VL;
    tr->side = -mover;
    tr->move_no += 1;
  } else {
    reset_tree(tr, b, d.N, -mover, tr->move_no + 1);
  }
}

__global__ void tree_sizes_kernel(MctsDev d, int32_t* nodes, int32_t* edges) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= d.trees) return;
  nodes[t] = d.tree[t].node_count;
  edges[t] = d.tree[t].edge_count;
}

// ---------------- chess (game kChess) ----------------
// The same waves on chess positions.  A warp per tree picks each level's
// edge by PUCT over up to 218 edges (lane j % 32 scores edge j; lowest index
// on ties, as above); lane 0 replays the path's actions on the root record,
// decides whether a new node ends the game (checkmate: a loss for its player
// to move; stalemate: a draw), and lists an unexpanded leaf's legal actions
// in generation order for the expansion.  Edges carry their action in pad[0].
// The end-of-game check of a new node and the leaf's legal list run after
// the wave's selections, a warp per leaf (chess_leaf_kernel): a new node
// is unexpanded, so it ends a selection whether or not the game ends there,
// and nothing in the selections depends on the check.

__device__ void chess_reset_tree(ChessTree* tr, const int8_t* rec, int side, int move_no) {
  for (int i = 0; i < 66; ++i) tr->rec[i] = rec[i];
  tr->side = (int8_t)(side >= 0 ? 1 : -1);
  tr->fe = -1;
  tr->meta = make_meta(0, 0, kNodeCreated);
  tr->n = 0;
  tr->vl = 0;
  tr->node_count = 1;
  tr->edge_count = 0;
  tr->move_no = move_no;
}

__global__ void chess_reset_kernel(MctsDev d, const int8_t* __restrict__ boards, const int8_t* __restrict__ side) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= d.trees) return;
  chess_reset_tree(d.ctree + t, boards + (size_t)t * 66, side[t], 0);
}

// PUCT score of an edge record (the select_tree arithmetic).
__device__ __forceinline__ float chess_puct(const MctsDev& d, int4 ra, float sq) {
  const int vlk = d.vl_k * ra.w;
  const int nev = ra.z + vlk;
  const float q = nev > 0 ? __fdiv_rn(__fsub_rn(__int_as_float(ra.y), (float)vlk), (float)nev) : 0.0f;
  const float u1 = __fmul_rn(d.c_puct, __int_as_float(ra.x));
  const float u2 = __fmul_rn(u1, sq);
  const float u3 = __fdiv_rn(u2, __fadd_rn(1.0f, (float)nev));
  return __fadd_rn(q, u3);
}

__device__ void chess_select_tree(const MctsDev& d, int t, int lane) {
  ChessTree* tr = d.ctree + t;
  MctsEdge* E = d.edges + (size_t)t * d.edge_cap;
  const int r_fe = tr->fe;
  const uint32_t r_meta = tr->meta;
  const int r_n = tr->n;
  int r_vl = tr->vl;
  int node_count = tr->node_count;
  for (int k = 0; k < d.leaves; ++k) {
    const size_t slot = (size_t)t * d.leaves + k;
    int* pe = d.path_edges + slot * kMctsMaxDepth;
    int fe = r_fe, ne = meta_edges(r_meta);
    uint32_t flags = meta_flags(r_meta);
    int np = r_n + d.vl_k * r_vl;
    r_vl += 1;
    chess::Pos p;
    chess::from_record(tr->rec, tr->side, p);
    int depth = 0;
    // an expanded node without edges (a root loaded in a finished game) is a leaf
    while ((flags & kNodeExpanded) && !(flags & kNodeTerminal) && ne > 0) {
      const float sq = __fsqrt_rn((float)np);
      float u = -INFINITY;
      int idx = 0x7fffffff;
      int4 ra = make_int4(0, 0, 0, 0), rb = make_int4(0, 0, 0, 0);
      for (int j = lane; j < ne; j += 32) {
        const int4* rec = (const int4*)(E + fe + j);
        const int4 a0 = rec[0], a1 = rec[1];
        float uj = chess_puct(d, a0, sq);
        if (uj != uj) uj = -INFINITY;  // a NaN prior or value sum: every lane still agrees on the pick
        if (uj > u || idx == 0x7fffffff) {
          u = uj;
          idx = j;
          ra = a0;
          rb = a1;
        }
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        const float uo = __shfl_xor_sync(kFull, u, o);
        const int io = __shfl_xor_sync(kFull, idx, o);
        if (uo > u || (uo == u && io < idx)) { u = uo; idx = io; }
      }
      const int src = idx & 31, e = fe + idx;
      const int c_nv = __shfl_sync(kFull, ra.z, src), c_vl = __shfl_sync(kFull, ra.w, src);
      const int c_fe = __shfl_sync(kFull, rb.x, src);
      const uint32_t c_meta = (uint32_t)__shfl_sync(kFull, rb.y, src);
      const int c_act = __shfl_sync(kFull, rb.z, src);
      uint32_t cflags = meta_flags(c_meta);
      if (!(cflags & kNodeCreated) && node_count >= d.node_cap) {
        if (lane == 0) set_err(d.err, kMctsNodeCap);
        break;
      }
      if (depth + 1 >= kMctsMaxDepth) {
        if (lane == 0) set_err(d.err, kMctsDepth);
        break;
      }
      if (lane == 0) {
        E[e].VL = c_vl + 1;
        pe[depth] = e;
      }
      chess::apply(p, chess::decode_action(p, c_act));
      ++depth;
      if (!(cflags & kNodeCreated)) {  // a new node: counted; its game-end check follows in the leaf pass
        ++node_count;
        cflags = kNodeCreated;
        if (lane == 0) E[e].meta = make_meta(0, 0, cflags);
      }
      flags = cflags;
      fe = c_fe;
      ne = meta_edges(c_meta);
      np = c_nv + d.vl_k * c_vl;
    }
    if (lane == 0) {
      d.path_len[slot] = depth;
      d.leaf_side[slot] = p.side;
      chess::to_record(p, d.leaf_board + slot * 66);
    }
  }
  if (lane == 0) {
    tr->vl = r_vl;
    tr->node_count = node_count;
  }
}

__device__ void chess_backup_tree(const MctsDev& d, const float* __restrict__ pi, const float* __restrict__ value,
                                  int t, int lane) {
  ChessTree* tr = d.ctree + t;
  MctsEdge* E = d.edges + (size_t)t * d.edge_cap;
  int r_fe = tr->fe;
  uint32_t r_meta = tr->meta;
  int r_n = tr->n, r_vl = tr->vl, edge_count = tr->edge_count;
  const int move_no = tr->move_no;
  for (int k = 0; k < d.leaves; ++k) {
    const size_t slot = (size_t)t * d.leaves + k;
    const int* pe = d.path_edges + slot * kMctsMaxDepth;
    const int len = d.path_len[slot];
    const int e0 = lane < len ? pe[lane] : -1;
    const int e1 = lane + 32 < len ? pe[lane + 32] : -1;
    const int le = len > 0 ? __shfl_sync(kFull, len - 1 < 32 ? e0 : e1, (len - 1) & 31) : -1;
    uint32_t lmeta = r_meta;
    if (len > 0 && lane == 0) lmeta = E[le].meta;
    lmeta = __shfl_sync(kFull, lmeta, 0);
    const uint32_t lflags = meta_flags(lmeta);
    float val;
    if (lflags & kNodeTerminal) {
      val = (lflags & kNodeLoss) ? -1.0f : 0.0f;
    } else {
      val = value[slot];
      if (!(lflags & kNodeExpanded)) {
        const float* p = pi + slot * d.A;
        const int16_t* la = d.leaf_actions + slot * kChessMaxLegal;
        const int cnt = d.leaf_count[slot];
        float sum = 0.0f;
        int fe = 0;
        if (lane == 0) {
          for (int j = 0; j < cnt; ++j) sum = __fadd_rn(sum, p[la[j]]);
          fe = edge_count;
          if (fe + cnt > d.edge_cap) {
            set_err(d.err, kMctsEdgeCap);
            fe = -1;
          } else {
            edge_count = fe + cnt;
          }
        }
        sum = __shfl_sync(kFull, sum, 0);
        fe = __shfl_sync(kFull, fe, 0);
        if (fe >= 0) {
          for (int j = lane; j < cnt; j += 32) {
            const int a = la[j];
            int4* rec = (int4*)(E + fe + j);
            rec[0] = make_int4(__float_as_int(__fdiv_rn(p[a], sum)), __float_as_int(0.0f), 0, 0);
            rec[1] = make_int4(-1, (int)make_meta(0, 0, 0), a, 0);
          }
          __syncwarp();
          if (lane == 0) {
            if (d.dir_eps > 0.0f && len == 0 && cnt > 0) {
              // root noise, P = (1 - eps) P + eps Dir(alpha); the gammas are
              // drawn twice (the sum, then each share) instead of stored
              float gs = 0.0f;
              for (int j = 0; j < cnt; ++j)
                gs += sample_gamma(d.dir_alpha, d.seed, (unsigned long long)t, ((unsigned long long)move_no << 8) | j);
              for (int j = 0; j < cnt; ++j) {
                const float g =
                    sample_gamma(d.dir_alpha, d.seed, (unsigned long long)t, ((unsigned long long)move_no << 8) | j);
                E[fe + j].P = (1.0f - d.dir_eps) * E[fe + j].P + d.dir_eps * (gs > 0.0f ? g / gs : 1.0f / cnt);
              }
            }
            const uint32_t nm = make_meta(0, cnt, lflags | kNodeExpanded);
            if (len > 0) {
              E[le].child_fe = fe;
              E[le].meta = nm;
            } else {
              r_fe = fe;
              r_meta = nm;
            }
          }
          r_fe = __shfl_sync(kFull, r_fe, 0);
          r_meta = __shfl_sync(kFull, r_meta, 0);
        }
      }
    }
    __syncwarp();
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int i = lane + 32 * h, e = h ? e1 : e0;
      if (i < len) {
        const float x = ((len - 1 - i) & 1) ? val : -val;
        int4* rec = (int4*)(E + e);
        int4 s = rec[0];
        s.y = __float_as_int(__fadd_rn(__int_as_float(s.y), x));
        s.z += 1;
        s.w -= 1;
        rec[0] = s;
      }
    }
    r_n += 1;
    r_vl -= 1;
    __syncwarp();
  }
  if (lane == 0) {
    tr->fe = r_fe;
    tr->meta = r_meta;
    tr->n = r_n;
    tr->vl = r_vl;
    tr->edge_count = edge_count;
  }
}

// The wave's leaf pass, a warp per selection: a node created in this wave
// gets its game-end check (checkmate: a loss for its player to move;
// stalemate: a draw), and a non-terminal unexpanded leaf its legal actions
// in generation order.  Lane l generates and tests the moves of squares l
// and l + 32 (at most 27 per piece), and a prefix sum over the lanes places
// them: squares ascending, each square's moves in piece_moves' order, as
// legal_moves lists them.  Two selections that end on the same new node
// write the same flags.
__global__ void chess_leaf_kernel(MctsDev d) {
  const int slot = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (slot >= d.trees * d.leaves) return;  // whole warps
  const int t = slot / d.leaves, len = d.path_len[slot];
  MctsEdge* E = d.edges + (size_t)t * d.edge_cap;
  const int le = len > 0 ? d.path_edges[(size_t)slot * kMctsMaxDepth + len - 1] : -1;
  uint32_t flags = meta_flags(len > 0 ? E[le].meta : d.ctree[t].meta);
  chess::Pos p;
  chess::from_record(d.leaf_board + (size_t)slot * 66, d.leaf_side[slot], p);
  const bool fresh = len > 0 && !(flags & kNodeChecked);  // created this wave, so not expanded
  const bool need_list = fresh || (!(flags & kNodeTerminal) && !(flags & kNodeExpanded));
  int c = 0, ks = -1;
  if (need_list) {
    const int king = p.side * chess::kKing;
    const unsigned b0 = __ballot_sync(kFull, p.sq[lane] == king), b1 = __ballot_sync(kFull, p.sq[lane + 32] == king);
    ks = b0 ? __ffs(b0) - 1 : b1 ? 31 + __ffs(b1) : -1;  // the lowest square, as king_square
    int16_t* la = d.leaf_actions + (size_t)slot * kChessMaxLegal;
    int base = 0;
    for (int h = 0; h < 2; ++h) {
      chess::Move mv[28];
      const int nm = chess::piece_moves(p, lane + 32 * h, mv, 28);
      int nl = 0;
      for (int k = 0; k < nm; ++k)
        if (chess::move_is_legal(p, mv[k], ks)) mv[nl++] = mv[k];
      int inc = nl;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(kFull, inc, o);
        if (lane >= o) inc += y;
      }
      const int off = base + inc - nl;
      for (int k = 0; k < nl; ++k)
        if (off + k < kChessMaxLegal) la[off + k] = (int16_t)chess::encode_action(mv[k]);
      base += __shfl_sync(kFull, inc, 31);
    }
    c = base < kChessMaxLegal ? base : kChessMaxLegal;
  }
  if (fresh) {
    const int oc = c > 0 ? 0 : (ks >= 0 && chess::attacked(p, ks, -p.side)) ? -1 : 2;
    flags |= kNodeChecked | (oc != 0 ? kNodeTerminal : 0u) | (oc == -1 ? kNodeLoss : 0u);
    if (lane == 0) E[le].meta = make_meta(0, 0, flags);
  }
  const bool term = (flags & kNodeTerminal) != 0;
  if (lane == 0) {
    d.leaf_terminal[slot] = term ? 1 : 0;
    d.leaf_count[slot] = term ? 0 : c;
  }
}

__global__ void chess_select_kernel(MctsDev d) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (t < d.trees) chess_select_tree(d, t, threadIdx.x & 31);
}

__global__ void chess_backup_kernel(MctsDev d, const float* __restrict__ pi, const float* __restrict__ value) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (t < d.trees) chess_backup_tree(d, pi, value, t, threadIdx.x & 31);
}

__global__ void chess_backup_select_kernel(MctsDev d, const float* __restrict__ pi, const float* __restrict__ value) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (t >= d.trees) return;
  chess_backup_tree(d, pi, value, t, threadIdx.x & 31);
  __syncwarp();
  chess_select_tree(d, t, threadIdx.x & 31);
}

__global__ void chess_root_visits_kernel(MctsDev d, int32_t* __restrict__ visits, float* __restrict__ wsum) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= d.trees) return;
  const ChessTree* tr = d.ctree + t;
  const MctsEdge* E = d.edges + (size_t)t * d.edge_cap;
  for (int a = 0; a < d.A; ++a) {
    visits[(size_t)t * d.A + a] = 0;
    if (wsum) wsum[(size_t)t * d.A + a] = 0.0f;
  }
  if (!(meta_flags(tr->meta) & kNodeExpanded)) return;
  const int fe = tr->fe, ne = meta_edges(tr->meta);
  for (int k = 0; k < ne; ++k) {
    const MctsEdge& e = E[fe + k];
    visits[(size_t)t * d.A + e.pad[0]] = e.Nv;
    if (wsum) wsum[(size_t)t * d.A + e.pad[0]] = e.W;
  }
}

// choose_kernel's rule on chess roots (edges in generation order); an
// unexpanded root plays its first legal action (0 if it has none).
__global__ void chess_choose_kernel(MctsDev d, int temp_moves, int32_t* __restrict__ actions) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= d.trees) return;
  const ChessTree* tr = d.ctree + t;
  const MctsEdge* E = d.edges + (size_t)t * d.edge_cap;
  const int fe = tr->fe, ne = (meta_flags(tr->meta) & kNodeExpanded) ? meta_edges(tr->meta) : 0;
  int pick = -1;
  if (ne > 0) {
    long long total = 0;
    int best = 0;
    for (int k = 0; k < ne; ++k) {
      const int nv = E[fe + k].Nv;
      total += nv;
      if (nv > E[fe + best].Nv) best = k;
    }
    pick = best;
    if (tr->move_no < temp_moves && total > 0) {
      const unsigned long long h = rng64(d.seed, (unsigned long long)t, (unsigned long long)tr->move_no, 0xC4);
      const long long x = (long long)(((h >> 32) * (unsigned long long)total) >> 32);
      long long cum = 0;
      for (int k = 0; k < ne; ++k) {
        cum += E[fe + k].Nv;
        if (cum > x) { pick = k; break; }
      }
    }
  }
  if (pick >= 0) {
    actions[t] = E[fe + pick].pad[0];
  } else {
    chess::Pos p;
    chess::from_record(tr->rec, tr->side, p);
    chess::Move ms[256];
    actions[t] = chess::legal_moves_inplace(p, ms) > 0 ? chess::encode_action(ms[0]) : 0;
  }
}

// play_kernel's rule on chess roots: the action is checked against the
// legal moves (an illegal one ends the game as a draw); a finished game
// (checkmate or stalemate after the move) restarts from the initial
// position with white to move.
__global__ void chess_play_kernel(MctsDev d, const int32_t* __restrict__ actions, int reserve,
                                  int8_t* __restrict__ done) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= d.trees) return;
  ChessTree* tr = d.ctree + t;
  const MctsEdge* E = d.edges + (size_t)t * d.edge_cap;
  const int a = actions[t];
  const MctsEdge* ce = nullptr;
  if (meta_flags(tr->meta) & kNodeExpanded) {
    const int fe = tr->fe, ne = meta_edges(tr->meta);
    for (int k = 0; k < ne; ++k)
      if (E[fe + k].pad[0] == a && (meta_flags(E[fe + k].meta) & kNodeCreated)) ce = E + fe + k;
  }
  chess::Pos p;
  chess::from_record(tr->rec, tr->side, p);
  chess::Move m, ms[256];
  int oc = 2;
  if (chess::find_action_with(p, a, &m, ms)) {
    chess::apply(p, m);
    oc = chess::outcome_with(p, ms);
  }
  if (done) done[t] = (int8_t)(oc != 0);
  int8_t rec[66];
  if (oc != 0) {
    chess::Pos s0;
    chess::start_pos(s0);
    chess::to_record(s0, rec);
    chess_reset_tree(tr, rec, 1, 0);
  } else if (ce && tr->node_count + reserve <= d.node_cap) {
    chess::to_record(p, tr->rec);
    tr->side = p.side;
    tr->fe = ce->child_fe;
    tr->meta = make_meta(0, meta_edges(ce->meta), meta_flags(ce->meta));
    tr->n = ce->Nv;
    tr->vl = ce->VL;
    tr->move_no += 1;
  } else {
    chess::to_record(p, rec);
    chess_reset_tree(tr, rec, p.side, tr->move_no + 1);
  }
}

__global__ void chess_tree_sizes_kernel(MctsDev d, int32_t* nodes, int32_t* edges) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= d.trees) return;
  nodes[t] = d.ctree[t].node_count;
  edges[t] = d.ctree[t].edge_count;
}

inline int blocks_for(int n, int per) { return (n + per - 1) / per; }

}  // namespace

cudaError_t mcts_launch_reset(const MctsDev& d, const int8_t* boards, const int8_t* side, cudaStream_t s) {
  if (d.game == kChess) chess_reset_kernel<<<blocks_for(d.trees, 128), 128, 0, s>>>(d, boards, side);
  else reset_kernel<<<blocks_for(d.trees, 128), 128, 0, s>>>(d, boards, side);
  return cudaGetLastError();
}

cudaError_t mcts_launch_select(const MctsDev& d, cudaStream_t s) {
  if (d.game == kChess) {
    chess_select_kernel<<<blocks_for(d.trees, 4), 128, 0, s>>>(d);
    chess_leaf_kernel<<<blocks_for(d.trees * d.leaves, 4), 128, 0, s>>>(d);
  } else select_kernel<<<blocks_for(d.trees, 4), 128, 0, s>>>(d);
  return cudaGetLastError();
}

cudaError_t mcts_launch_backup(const MctsDev& d, const float* pi, const float* v, cudaStream_t s) {
  if (d.game == kChess) chess_backup_kernel<<<blocks_for(d.trees, 4), 128, 0, s>>>(d, pi, v);
  else backup_kernel<<<blocks_for(d.trees, 4), 128, 0, s>>>(d, pi, v);
  return cudaGetLastError();
}

cudaError_t mcts_launch_backup_select(const MctsDev& d, const float* pi, const float* v, cudaStream_t s) {
  if (d.game == kChess) {
    chess_backup_select_kernel<<<blocks_for(d.trees, 4), 128, 0, s>>>(d, pi, v);
    chess_leaf_kernel<<<blocks_for(d.trees * d.leaves, 4), 128, 0, s>>>(d);
  } else backup_select_kernel<<<blocks_for(d.trees, 4), 128, 0, s>>>(d, pi, v);
  return cudaGetLastError();
}

cudaError_t mcts_launch_root_visits(const MctsDev& d, int32_t* visits, float* wsum, cudaStream_t s) {
  if (d.game == kChess) chess_root_visits_kernel<<<blocks_for(d.trees, 128), 128, 0, s>>>(d, visits, wsum);
  else root_visits_kernel<<<blocks_for(d.trees, 128), 128, 0, s>>>(d, visits, wsum);
  return cudaGetLastError();
}

cudaError_t mcts_launch_choose(const MctsDev& d, int temp_moves, int32_t* actions, cudaStream_t s) {
  if (d.game == kChess) chess_choose_kernel<<<blocks_for(d.trees, 128), 128, 0, s>>>(d, temp_moves, actions);
  else choose_kernel<<<blocks_for(d.trees, 128), 128, 0, s>>>(d, temp_moves, actions);
  return cudaGetLastError();
}

cudaError_t mcts_launch_play(const MctsDev& d, const int32_t* actions, int reserve, int8_t* done, cudaStream_t s) {
  if (d.game == kChess) chess_play_kernel<<<blocks_for(d.trees, 128), 128, 0, s>>>(d, actions, reserve, done);
  else play_kernel<<<blocks_for(d.trees, 128), 128, 0, s>>>(d, actions, reserve, done);
  return cudaGetLastError();
}

cudaError_t mcts_launch_tree_sizes(const MctsDev& d, int32_t* nodes, int32_t* edges, cudaStream_t s) {
  if (d.game == kChess) chess_tree_sizes_kernel<<<blocks_for(d.trees, 128), 128, 0, s>>>(d, nodes, edges);
  else tree_sizes_kernel<<<blocks_for(d.trees, 128), 128, 0, s>>>(d, nodes, edges);
  return cudaGetLastError();
}

}  // namespace gz
