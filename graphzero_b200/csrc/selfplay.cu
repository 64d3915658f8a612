// Self-play episodes and arena games on top of the batched search.
//
// Self-play: every tree of a search handle plays games back to back; each move records the root position and
// its visit-count policy, and when a game ends its examples get the outcome
// and are copied, in a fixed order, to an output buffer of TrainingExample
// records.
//
// Reference: parallel_self_play_kernel and execute_self_play
// (self_play/self_play.cu:75-145, 403-472): per move, simulations, the
// policy N^(1/T) (mcts_get_policy, 645-662), the example (board, pi), the
// chosen move, the next state, and at the game's end v = the outcome for each
// example.  Differences, all deliberate:
//   * the stored board is the canonical form (board x player to move,
//     games/connect4/connect4.cu:89-93), so every example is seen from the
//     player to move, and v is the outcome for that player (+1 win, -1 loss,
//     0 draw); the reference stores the raw board and signs v by the parity of
//     the move index (self_play.cu:438-447), from a game-end test of the
//     player who did not just move;
//   * after temp_moves moves the policy is one-hot on the most visited move
//     (lowest action on ties), the limit of the reference's T = 1e-3;
//   * games never exceed the board's number of cells, so no forced draw at
//     MAX_GAME_LENGTH (self_play.cu:457-465) is needed.
//
// Arena (arena/arena.cu:31-106 with the NNet player of
// players/players.cu:96-104): games between two networks, each move searched
// from a fresh root by the side to move's network, the most visited move
// played; the helper kernels here merge the two networks' leaf evaluations
// per tree and apply the moves.
#include <cuda_runtime.h>
#include <stdint.h>

#include "gz_games.h"
#include "gz_mcts.h"

namespace gz {
namespace {

// The root's expanded edges: visit counts -> policy over actions (zeroed
// elsewhere).  T = 1 while move_no < temp_moves: N_a / sum N; afterwards
// one-hot on the most visited action (the first edge, i.e. the lowest
// action, on ties).
__device__ void root_policy(const MctsDev& d, int t, int temp_moves, float* pi) {
  const MctsTree* tr = d.tree + t;
  const MctsEdge* E = d.edges + (size_t)t * d.edge_cap;
  for (int a = 0; a < d.A; ++a) pi[a] = 0.0f;
  if (!(meta_flags(tr->meta) & kNodeExpanded)) return;
  const int fe = tr->fe, ne = meta_edges(tr->meta);
  long long total = 0;
  int best = 0;
  for (int k = 0; k < ne; ++k) {
    const int nv = E[fe + k].Nv;
    total += nv;
    if (nv > E[fe + best].Nv) best = k;
  }
  if (ne == 0) return;
  if (tr->move_no < temp_moves && total > 0) {
    for (int k = 0; k < ne; ++k) pi[meta_action(E[fe + k].meta)] = (float)E[fe + k].Nv / (float)total;
  } else {
    pi[meta_action(E[fe + best].meta)] = 1.0f;
  }
}

__global__ void record_kernel(MctsDev d, SelfPlayDev s, int temp_moves) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= d.trees) return;
  const int k = s.log_len[t];
  if (k >= s.max_moves) {  // cannot happen for games of at most max_moves plies
    atomicExch(s.overflow, 1);
    return;
  }
  const size_t slot = (size_t)t * s.max_moves + k;
  const MctsTree* tr = d.tree + t;
  const int side = tr->side;
  for (int i = 0; i < d.N; ++i) s.log_board[slot * d.N + i] = (int8_t)(tr->board[i] * side);
  root_policy(d, t, temp_moves, s.log_pi + slot * d.A);
  s.log_side[slot] = (int8_t)side;
  s.log_len[t] = k + 1;
}

// Outcome of the chosen move (before play_kernel applies it): a game that
// ends gets its examples' values and its length in fin_len.
__global__ void finish_kernel(MctsDev d, SelfPlayDev s, const int32_t* __restrict__ actions) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= d.trees) return;
  s.fin_len[t] = 0;
  const MctsTree* tr = d.tree + t;
  int8_t b[kMctsBoardStride];
  for (int i = 0; i < kMctsBoardStride; ++i) b[i] = tr->board[i];
  const int mover = tr->side;
  const int sq = apply_action(d.game, b, actions[t], mover);
  const int oc = sq < 0 ? 2 : outcome_after(d.game, b, sq, mover);
  if (oc == 0) return;
  const float z = oc == 1 ? 1.0f : 0.0f;  // for the mover
  const int n = s.log_len[t];
  for (int k = 0; k < n; ++k) {
    const size_t slot = (size_t)t * s.max_moves + k;
    s.log_v[slot] = s.log_side[slot] == mover ? z : -z;
  }
  s.fin_len[t] = n;
}

// Block-wide exclusive prefix sum (blockDim.x a multiple of 32, <= 1024).
__device__ int block_exclusive_sum(int x, int* total) {
  __shared__ int warp_sums[32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int incl = x;
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) warp_sums[w] = incl;
  __syncthreads();
  if (w == 0) {
    int v = lane < nw ? warp_sums[lane] : 0;
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += y;
    }
    if (lane < nw) warp_sums[lane] = v;  // inclusive over warps
  }
  __syncthreads();
  const int before = (w > 0 ? warp_sums[w - 1] : 0) + incl - x;
  *total = warp_sums[nw - 1];
  __syncthreads();
  return before;
}

// One block: the games that ended this move, in tree order, appended to the
// output as TrainingExample records (board and pi zero-padded to 64).
__global__ void emit_kernel(MctsDev d, SelfPlayDev s) {
  __shared__ int base_ex, base_games, first_lost;
  if (threadIdx.x == 0) {
    base_ex = *s.out_count;
    base_games = *s.games_done;
    first_lost = s.out_cap;  // where the first game that did not fit would have gone
  }
  __syncthreads();
  for (int t0 = 0; t0 < d.trees; t0 += blockDim.x) {
    const int t = t0 + threadIdx.x;
    const int n = t < d.trees ? s.fin_len[t] : 0;
    int tot_ex = 0, tot_games = 0;
    const int off = block_exclusive_sum(n, &tot_ex);
    block_exclusive_sum(n > 0 ? 1 : 0, &tot_games);
    if (n > 0) {
      const int dst = base_ex + off;
      if (dst + n > s.out_cap) {
        atomicExch(s.overflow, 2);
        atomicMin(&first_lost, dst);
      } else {
        for (int k = 0; k < n; ++k) {
          const size_t slot = (size_t)t * s.max_moves + k;
          gz_train_example* e = s.out + dst + k;
          for (int i = 0; i < GZ_EXAMPLE_CELLS; ++i) e->board[i] = i < d.N ? (int32_t)s.log_board[slot * d.N + i] : 0;
          for (int a = 0; a < GZ_EXAMPLE_CELLS; ++a) e->pi[a] = a < d.A ? s.log_pi[slot * d.A + a] : 0.0f;
          e->v = s.log_v[slot];
        }
      }
      s.log_len[t] = 0;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      base_ex += tot_ex;
      base_games += tot_games;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    // after an overflow the buffer holds the games before the first one that
    // did not fit (later games that would have fitted are dropped with it)
    *s.out_count = base_ex < first_lost ? base_ex : first_lost;
    *s.games_done = base_games;
  }
}

// Arena: per leaf slot, the evaluation of the network that searches at the
// slot's tree (net A where a_moves[tree], else net B).
__global__ void arena_merge_kernel(int n_leaves, int leaves_per_tree, int A, const int8_t* __restrict__ a_moves,
                                   const float* __restrict__ pi_a, const float* __restrict__ v_a,
                                   const float* __restrict__ pi_b, const float* __restrict__ v_b,
                                   float* __restrict__ pi, float* __restrict__ v) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= n_leaves) return;
  const bool a = a_moves[k / leaves_per_tree] != 0;
  for (int j = 0; j < A; ++j) pi[(size_t)k * A + j] = a ? pi_a[(size_t)k * A + j] : pi_b[(size_t)k * A + j];
  v[k] = a ? v_a[k] : v_b[k];
}

// Arena: the chosen moves applied to the games in play.  A game that ends
// records its result (1 = net A won, 2 = net B won, 3 = draw) and goes back
// to the empty board (searched but no longer played); otherwise the side to
// move flips and so does which network moves.
__global__ void arena_play_kernel(int game, int trees, int N, int8_t* __restrict__ boards, int8_t* __restrict__ side,
                                  int8_t* __restrict__ a_moves, int8_t* __restrict__ active,
                                  const int32_t* __restrict__ actions, int8_t* __restrict__ result,
                                  int* __restrict__ n_active) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= trees || !active[t]) return;
  int8_t b[kMctsBoardStride];
  for (int i = 0; i < N; ++i) b[i] = boards[(size_t)t * N + i];
  const int mover = side[t];
  const int sq = apply_action(game, b, actions[t], mover);
  const int oc = sq < 0 ? 2 : outcome_after(game, b, sq, mover);
  if (oc != 0) {
    result[t] = (int8_t)(oc == 2 ? 3 : (a_moves[t] ? 1 : 2));
    active[t] = 0;
    for (int i = 0; i < N; ++i) boards[(size_t)t * N + i] = 0;
    side[t] = 1;
    return;
  }
  for (int i = 0; i < N; ++i) boards[(size_t)t * N + i] = b[i];
  side[t] = (int8_t)(-mover);
  a_moves[t] = (int8_t)!a_moves[t];
  atomicAdd(n_active, 1);
}

}  // namespace

cudaError_t arena_launch_merge(int n_leaves, int leaves_per_tree, int A, const int8_t* a_moves, const float* pi_a,
                               const float* v_a, const float* pi_b, const float* v_b, float* pi, float* v,
                               cudaStream_t st) {
  arena_merge_kernel<<<(n_leaves + 255) / 256, 256, 0, st>>>(n_leaves, leaves_per_tree, A, a_moves, pi_a, v_a, pi_b,
                                                             v_b, pi, v);
  return cudaGetLastError();
}

cudaError_t arena_launch_play(int game, int trees, int N, int8_t* boards, int8_t* side, int8_t* a_moves,
                              int8_t* active, const int32_t* actions, int8_t* result, int* n_active,
                              cudaStream_t st) {
  arena_play_kernel<<<(trees + 127) / 128, 128, 0, st>>>(game, trees, N, boards, side, a_moves, active, actions,
                                                          result, n_active);
  return cudaGetLastError();
}

cudaError_t selfplay_launch_record(const MctsDev& d, const SelfPlayDev& s, int temp_moves, cudaStream_t st) {
  record_kernel<<<(d.trees + 127) / 128, 128, 0, st>>>(d, s, temp_moves);
  return cudaGetLastError();
}

cudaError_t selfplay_launch_finish(const MctsDev& d, const SelfPlayDev& s, const int32_t* actions, cudaStream_t st) {
  finish_kernel<<<(d.trees + 127) / 128, 128, 0, st>>>(d, s, actions);
  return cudaGetLastError();
}

cudaError_t selfplay_launch_emit(const MctsDev& d, const SelfPlayDev& s, cudaStream_t st) {
  emit_kernel<<<1, 1024, 0, st>>>(d, s);
  return cudaGetLastError();
}

}  // namespace gz
