// Device-side state of the batched PUCT search.
//
// Every tree owns one contiguous pool of edge records, so a warp walking its
// tree touches one region of memory (a few pages, not one page per field
// array).  A node exists only through the edge that leads to it: that edge
// carries the child's statistics (its visit and in-flight counts are the
// edge's, since every path through the child passes the edge) and, once the
// child is expanded, where the child's own edges start and how many there
// are.  A selection level is therefore one round of loads: the current node's
// edges.  The root's fields live in the per-tree record, with its position;
// positions below the root are not stored (a selection replays its actions
// on the root position in registers).  This replaces the reference's
// MCTSNode with fixed 218-entry child arrays and child pointers
// (mcts/mcts.cuh:25-36).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/graphzero_b200.h"

namespace gz {

constexpr int kMctsBoardStride = 48;  // bytes per stored position (>= 42, 16-aligned)
constexpr int kMctsMaxDepth = 48;     // >= longest game (42 plies) + 1

// Child flags (MctsEdge::meta bits 16-23, MctsTree::meta likewise).
enum : uint32_t {
  kNodeCreated = 1u,   // the child exists (counts against node_capacity)
  kNodeExpanded = 2u,  // its edges exist
  kNodeTerminal = 4u,  // the game is over at the child
  kNodeLoss = 8u,      // terminal with a loss for the child's player to move (value -1; else 0)
  kNodeChecked = 16u,  // chess: the game-end check of the node has run (the wave's leaf pass)
};

__host__ __device__ __forceinline__ uint32_t meta_action(uint32_t m) { return m & 0xffu; }
__host__ __device__ __forceinline__ int meta_edges(uint32_t m) { return (int)((m >> 8) & 0xffu); }
__host__ __device__ __forceinline__ uint32_t meta_flags(uint32_t m) { return (m >> 16) & 0xffu; }

struct alignas(16) MctsEdge {  // 32 bytes: one per (expanded node, legal action)
  float P;                     // prior (legal-renormalised, root noise mixed in)
  float W;                     // value sum, from the view of the player to move at the parent
  int32_t Nv;                  // completed visits (= the child's)
  int32_t VL;                  // selections in flight (= the child's)
  int32_t child_fe;            // the child's first edge, once expanded
  uint32_t meta;               // action | child edge count << 8 | child flags << 16
  int32_t pad[2];
};
static_assert(sizeof(MctsEdge) == 32, "edge record");

struct alignas(16) MctsTree {  // 128 bytes per tree
  int8_t board[kMctsBoardStride];  // root position
  int32_t fe;                      // root's first edge
  uint32_t meta;                   // root's edge count << 8 | flags << 16
  int32_t n, vl;                   // root's completed visits and selections in flight
  int32_t node_count, edge_count;  // pool use (nodes are counted, not stored)
  int32_t move_no;                 // moves played since the game started
  int32_t side;                    // player to move at the root
  int32_t pad[12];
};
static_assert(sizeof(MctsTree) == 128, "tree record");

// Chess trees (game kChess) keep the root as the 66-byte record plus the
// side to move, and their edges carry the action index (from * 73 + t, up
// to 4671) in pad[0]; meta's action byte is unused.  Edge counts (<= 218
// legal moves) still fit meta's 8 bits.
struct alignas(16) ChessTree {  // 128 bytes per tree
  int8_t rec[66];                // root position (squares, castling rights, en-passant square)
  int8_t side;                   // player to move at the root
  int8_t pad0;
  int32_t fe;                    // root's first edge
  uint32_t meta;                 // root's edge count << 8 | flags << 16
  int32_t n, vl;
  int32_t node_count, edge_count;
  int32_t move_no;
  int32_t pad[8];
};
static_assert(sizeof(ChessTree) == 128, "chess tree record");
constexpr int kChessMaxLegal = 256;  // legal-action list length per leaf (<= 218 in chess)

struct MctsDev {
  int game, trees, leaves, vl_k, node_cap, edge_cap, N, A;
  int board_bytes;  // bytes per stored position (N, 66 for chess)
  float c_puct, dir_alpha, dir_eps;
  unsigned long long seed;
  MctsTree* tree;   // [trees]
  MctsEdge* edges;  // [trees][edge_cap]
  // selections of the current wave, slot = tree * leaves + k
  int* path_edges;     // [slots][kMctsMaxDepth] edge chosen at each level
  int* path_len;       // [slots]
  uint32_t* leaf_legal;  // [slots] legal actions at the leaf (bit a)
  // leaf batch (network input) [slots]
  int8_t* leaf_board;  // [slots][N]
  int8_t* leaf_side;
  int8_t* leaf_terminal;
  int* err;  // first error code seen by a kernel (0 = none)
  // chess only
  ChessTree* ctree;       // [trees]
  int16_t* leaf_actions;  // [slots][kChessMaxLegal] legal actions at the leaf, generation order
  int32_t* leaf_count;    // [slots]
};

enum MctsErr : int { kMctsOk = 0, kMctsNodeCap = 1, kMctsEdgeCap = 2, kMctsDepth = 3 };

cudaError_t mcts_launch_reset(const MctsDev& d, const int8_t* boards, const int8_t* side, cudaStream_t s);
cudaError_t mcts_launch_select(const MctsDev& d, cudaStream_t s);
cudaError_t mcts_launch_backup(const MctsDev& d, const float* pi, const float* v, cudaStream_t s);
// backup of the current wave, then the next wave's selections (one launch)
cudaError_t mcts_launch_backup_select(const MctsDev& d, const float* pi, const float* v, cudaStream_t s);
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
