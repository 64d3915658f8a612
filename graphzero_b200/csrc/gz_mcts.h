// Device-side state of the batched PUCT search (structure of arrays).
//
// Every tree owns a private pool of nodes and edges; indices are local to the
// tree (global = tree * cap + local).  A node keeps its position so a leaf can
// be encoded without replaying the path.  This replaces the reference's
// MCTSNode with fixed 218-entry child arrays and child pointers
// (mcts/mcts.cuh:25-36).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/graphzero_b200.h"

namespace gz {

constexpr int kMctsBoardStride = 48;  // bytes per stored position (>= 42, 16-aligned)
constexpr int kMctsMaxDepth = 48;     // >= longest game (42 plies) + 1

struct MctsDev {
  int game, trees, leaves, vl_k, node_cap, edge_cap, N, A;
  float c_puct, dir_alpha, dir_eps;
  unsigned long long seed;
  // nodes [trees * node_cap]
  int* n;           // completed backups through the node
  int* vl;          // selections in flight through the node
  int* first_edge;  // local edge index of the first child edge
  int8_t* n_edges;
  int8_t* side;     // player to move at the node
  int8_t* expanded;
  int8_t* terminal;
  float* term_value;  // value for the player to move at a terminal node
  int8_t* board;      // [trees * node_cap][kMctsBoardStride]
  // edges [trees * edge_cap]
  float* P;
  float* W;  // value sum from the perspective of the player to move at the parent
  int* Nv;   // visit count
  int* VL;   // virtual visits in flight
  int* child;
  int8_t* action;
  // per tree
  int* root;
  int* node_count;
  int* edge_count;
  int* move_no;
  // selection paths [trees][leaves][kMctsMaxDepth]
  int* path_nodes;
  int* path_edges;
  int* path_len;  // [trees][leaves]
  // leaf batch (network input) [trees * leaves]
  int8_t* leaf_board;  // [trees * leaves][N]
  int8_t* leaf_side;
  int8_t* leaf_terminal;
  int* err;  // first error code seen by a kernel (0 = none)
};

enum MctsErr : int { kMctsOk = 0, kMctsNodeCap = 1, kMctsEdgeCap = 2, kMctsDepth = 3 };

cudaError_t mcts_launch_reset(const MctsDev& d, const int8_t* boards, const int8_t* side, cudaStream_t s);
cudaError_t mcts_launch_select(const MctsDev& d, cudaStream_t s);
cudaError_t mcts_launch_backup(const MctsDev& d, const float* pi, const float* v, cudaStream_t s);
cudaError_t mcts_launch_root_visits(const MctsDev& d, int32_t* visits, float* wsum, cudaStream_t s);
cudaError_t mcts_launch_choose(const MctsDev& d, int temp_moves, int32_t* actions, cudaStream_t s);
cudaError_t mcts_launch_play(const MctsDev& d, const int32_t* actions, int reserve, int8_t* done, cudaStream_t s);
cudaError_t mcts_launch_tree_sizes(const MctsDev& d, int32_t* nodes, int32_t* edges, cudaStream_t s);

// Self-play bookkeeping (selfplay.cu): per-tree logs of the game in progress
// and the output buffer of finished examples.
struct SelfPlayDev {
  int max_moves;          // examples one game can produce (plies)
  int8_t* log_board;      // [trees][max_moves][N] canonical boards
  float* log_pi;          // [trees][max_moves][A]
  float* log_v;           // [trees][max_moves]
  int8_t* log_side;       // [trees][max_moves] player to move
  int* log_len;           // [trees] examples of the game in progress
  int* fin_len;           // [trees] examples of the game that ended this move (0 = none)
  gz_train_example* out;  // [out_cap]
  int out_cap;
  int* out_count;
  int* games_done;
  int* overflow;          // 1 = a game log overflowed, 2 = the output buffer did
};

// Per move, around mcts_launch_choose: record the roots, then (given the
// chosen actions, before mcts_launch_play) finish ended games and emit them.
cudaError_t selfplay_launch_record(const MctsDev& d, const SelfPlayDev& s, int temp_moves, cudaStream_t st);
cudaError_t selfplay_launch_finish(const MctsDev& d, const SelfPlayDev& s, const int32_t* actions, cudaStream_t st);
cudaError_t selfplay_launch_emit(const MctsDev& d, const SelfPlayDev& s, cudaStream_t st);

// Arena helpers (selfplay.cu): per-tree choice between two networks' leaf
// evaluations, and the moves applied to the games in play (result per tree:
// 1 = net A won, 2 = net B won, 3 = draw; n_active counts games still going).
cudaError_t arena_launch_merge(int n_leaves, int leaves_per_tree, int A, const int8_t* a_moves, const float* pi_a,
                               const float* v_a, const float* pi_b, const float* v_b, float* pi, float* v,
                               cudaStream_t st);
cudaError_t arena_launch_play(int game, int trees, int N, int8_t* boards, int8_t* side, int8_t* a_moves,
                              int8_t* active, const int32_t* actions, int8_t* result, int* n_active,
                              cudaStream_t st);

}  // namespace gz
