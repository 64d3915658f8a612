// Game geometry, rules and feature encoding shared by the host runtime and the
// device kernels of graphzero_b200.
//
// Board conventions follow the reference games:
//   * squares are row-major, node = row * cols + col
//     (games/connect4/connect4.cu:26-28, games/tictactoe/tictactoe.cu:24-31);
//   * cells hold {-1, 0, +1}; the first player is +1 and players alternate
//     (connect4.cu:22-34 sets next_player = -player);
//   * Connect4 action = column, a stone drops to the lowest empty row
//     (connect4.cu:22-34), a column is legal while its top cell is empty
//     (connect4.cu:36-40);
//   * chess squares are rank * 8 + file with piece codes +-1..6 for
//     P N B R Q K (games/chess/chess.cuh:11-21) and actions start * 73 + type
//     (games/chess/chess.cu:96-100,127-135).
//
// The reference dispatches rules through IGame function pointers that kernels
// cannot call (games/game.cuh:12-28); here rules are static inline functions
// specialised per game, callable from host and device alike.
#pragma once
#include <stddef.h>
#include <stdint.h>

#if defined(__CUDACC__)
#define GZ_HD __host__ __device__ __forceinline__
#define GZ_HDI __host__ __device__ inline  // larger host/device functions, inlined at the compiler's choice
#else
#define GZ_HD static inline
#define GZ_HDI inline
#endif

namespace gz {

constexpr int kHidden = 256;     // concat of 8 heads x 32 (networks/gat/gat.cu:705-707)
constexpr int kHeads = 8;
constexpr int kHeadDim = 32;
constexpr int kValueHidden = 64;
constexpr float kLeakySlope = 0.2f;  // networks/gat/gat.cu:715, config/config.json:28

enum GameId : int { kTicTacToe = 0, kConnect4 = 1, kChess = 2 };

// Static per-game sizes.  P is the per-node policy width, BOARD the number of
// bytes of one encoded position (chess adds a castling-rights byte and an
// en-passant square byte after the 64 squares).
template <int G> struct Traits;
template <> struct Traits<kTicTacToe> {
  static constexpr int N = 9, ROWS = 3, COLS = 3, A = 9, F = 4, L = 4, P = 1, BOARD = 9, NNZ = 49;
};
template <> struct Traits<kConnect4> {
  static constexpr int N = 42, ROWS = 6, COLS = 7, A = 7, F = 4, L = 6, P = 1, BOARD = 42, NNZ = 304;
};
template <> struct Traits<kChess> {
  static constexpr int N = 64, ROWS = 8, COLS = 8, A = 4672, F = 18, L = 8, P = 73, BOARD = 66, NNZ = 1856;
};

struct GameShape {
  int nodes, rows, cols, actions, features, layers, policy_out, board_bytes, nnz;
};

GZ_HD GameShape game_shape(int g) {
  GameShape s{};
  if (g == kTicTacToe) s = GameShape{9, 3, 3, 9, 4, 4, 1, 9, 49};
  else if (g == kConnect4) s = GameShape{42, 6, 7, 7, 4, 6, 1, 42, 304};
  else if (g == kChess) s = GameShape{64, 8, 8, 4672, 18, 8, 73, 66, 1856};
  return s;
}

// ---------------------------------------------------------------------------
// Board graph (static CSR, neighbours ascending, self loop included).
//   TicTacToe / Connect4: 8-neighbourhood (king moves) + self.
//   Chess: unobstructed queen lines + knight jumps + self; the geometry of the
//   reference's attack tables (games/chess/chess.cu:955-1008).
// Writes row_ptr[N+1] and col[nnz]; returns nnz.
// ---------------------------------------------------------------------------
GZ_HD bool graph_adjacent(int g, int rows, int cols, int i, int j) {
  int ri = i / cols, ci = i % cols, rj = j / cols, cj = j % cols;
  int dr = rj - ri, dc = cj - ci;
  int ar = dr < 0 ? -dr : dr, ac = dc < 0 ? -dc : dc;
  if (i == j) return true;
  if (g != kChess) return ar <= 1 && ac <= 1;
  if (dr == 0 || dc == 0 || ar == ac) return true;        // queen line
  return (ar == 1 && ac == 2) || (ar == 2 && ac == 1);    // knight
}

GZ_HD int build_graph_csr(int g, int* row_ptr, int* col) {
  GameShape s = game_shape(g);
  int nnz = 0;
  for (int i = 0; i < s.nodes; ++i) {
    row_ptr[i] = nnz;
    for (int j = 0; j < s.nodes; ++j)
      if (graph_adjacent(g, s.rows, s.cols, i, j)) col[nnz++] = j;
  }
  row_ptr[s.nodes] = nnz;
  return nnz;
}

// ---------------------------------------------------------------------------
// Node features.  TicTacToe / Connect4 (F = 4):
//   [empty, own, opponent, side-to-move-is-first-player]
// where own means board == side.  Chess (F = 18):
//   [0..5]  white P N B R Q K, [6..11] black P N B R Q K,
//   [12] white to move, [13..16] castling rights WK WQ BK BQ (bits 0..3 of
//   byte 64), [17] node is the en-passant target (byte 65, -1 = none).
// ---------------------------------------------------------------------------
GZ_HD void encode_node(int g, const int8_t* board, int side, int node, float* f) {
  if (g != kChess) {
    int v = board[node];
    f[0] = v == 0 ? 1.f : 0.f;
    f[1] = v == side ? 1.f : 0.f;
    f[2] = v == -side ? 1.f : 0.f;
    f[3] = side == 1 ? 1.f : 0.f;
    return;
  }
  int v = board[node];
  for (int k = 0; k < 18; ++k) f[k] = 0.f;
  if (v > 0) f[v - 1] = 1.f;
  if (v < 0) f[6 + (-v) - 1] = 1.f;
  f[12] = side == 1 ? 1.f : 0.f;
  int castle = (uint8_t)board[64];
  for (int b = 0; b < 4; ++b) f[13 + b] = (castle >> b) & 1 ? 1.f : 0.f;
  f[17] = board[65] == node ? 1.f : 0.f;
}

// ---------------------------------------------------------------------------
// Rules (TicTacToe, Connect4).  `moved` is the player who just placed a stone.
// ---------------------------------------------------------------------------
GZ_HD bool ttt_line_win(const int8_t* b, int p) {
  for (int i = 0; i < 3; ++i) {
    if (b[3 * i] == p && b[3 * i + 1] == p && b[3 * i + 2] == p) return true;
    if (b[i] == p && b[i + 3] == p && b[i + 6] == p) return true;
  }
  if (b[0] == p && b[4] == p && b[8] == p) return true;
  if (b[2] == p && b[4] == p && b[6] == p) return true;
  return false;
}

GZ_HD int c4_count_dir(const int8_t* b, int r, int c, int dr, int dc, int p) {
  int n = 0;
  for (int k = 1; k < 4; ++k) {
    int rr = r + k * dr, cc = c + k * dc;
    if (rr < 0 || rr >= 6 || cc < 0 || cc >= 7 || b[rr * 7 + cc] != p) break;
    ++n;
  }
  return n;
}

// Four in a row through (r, c) for player p.
GZ_HD bool c4_win_through(const int8_t* b, int r, int c, int p) {
  const int d[4][2] = {{0, 1}, {1, 0}, {1, 1}, {1, -1}};
  for (int k = 0; k < 4; ++k) {
    int n = 1 + c4_count_dir(b, r, c, d[k][0], d[k][1], p) + c4_count_dir(b, r, c, -d[k][0], -d[k][1], p);
    if (n >= 4) return true;
  }
  return false;
}

GZ_HD bool action_legal(int g, const int8_t* b, int a) {
  if (g == kConnect4) return a >= 0 && a < 7 && b[a] == 0;  // top cell empty
  return a >= 0 && a < 9 && b[a] == 0;
}

// Apply `a` for player p in place.  Returns the square written, or -1.
GZ_HD int apply_action(int g, int8_t* b, int a, int p) {
  if (g == kConnect4) {
    for (int r = 5; r >= 0; --r)
      if (b[r * 7 + a] == 0) { b[r * 7 + a] = (int8_t)p; return r * 7 + a; }
    return -1;
  }
  if (b[a] != 0) return -1;
  b[a] = (int8_t)p;
  return a;
}

// Outcome after player `moved` wrote `square`: 1 = mover won, 2 = draw
// (board full), 0 = game continues.
GZ_HD int outcome_after(int g, const int8_t* b, int square, int moved) {
  bool win = g == kConnect4 ? c4_win_through(b, square / 7, square % 7, moved) : ttt_line_win(b, moved);
  if (win) return 1;
  int n = g == kConnect4 ? 7 : 9;  // Connect4: full iff the top row is full
  for (int i = 0; i < n; ++i)
    if (b[i] == 0) return 0;
  return 2;
}

// ---------------------------------------------------------------------------
// Weight-blob layouts (fp32, contiguous, offsets in floats).
// GAT, per layer l (F_0 = game features, F_l = 256 afterwards):
//   W_l [F_l][256] (row = input feature), b_l [256], a_l [8 heads][2][32]
//   where a_l[h][0] scores the aggregating node i and a_l[h][1] the neighbour j
//   (the reference keeps [heads][2][hidden], networks/gat/gat.cu:62).
// Heads: w_pi [256][P], b_pi [P], W_v1 [256][64], b_v1 [64], w_v2 [64], b_v2 [1].
// ---------------------------------------------------------------------------
struct GatLayout {
  int L, F, P;
  size_t W[8], b[8], a[8];
  size_t w_pi, b_pi, W_v1, b_v1, w_v2, b_v2, total;
};

GZ_HD GatLayout gat_layout(int game) {
  GameShape s = game_shape(game);
  GatLayout t{};
  t.L = s.layers; t.F = s.features; t.P = s.policy_out;
  size_t o = 0;
  for (int l = 0; l < t.L; ++l) {
    int fin = l == 0 ? t.F : kHidden;
    t.W[l] = o; o += (size_t)fin * kHidden;
    t.b[l] = o; o += kHidden;
    t.a[l] = o; o += kHeads * 2 * kHeadDim;
  }
  t.w_pi = o; o += (size_t)kHidden * t.P;
  t.b_pi = o; o += t.P;
  t.W_v1 = o; o += (size_t)kHidden * kValueHidden;
  t.b_v1 = o; o += kValueHidden;
  t.w_v2 = o; o += kValueHidden;
  t.b_v2 = o; o += 1;
  t.total = o;
  return t;
}

// ResNet (Connect4, 128 channels, 10 blocks; the reference's tower at
// networks/resnet/resnet.cu:350-394 with a real residual add).  Conv weights are
// [Cout][ky][kx][Cin]; every BN is stored as gamma, beta, mean, var (each [C]).
//   stem conv 3->128, bn; blocks x10 {conv1, bn1, conv2, bn2};
//   policy conv 1x1 128->2 [2][128], bn(2), fc [84][7] (input index c*42+pos), fc_b [7];
//   value conv 1x1 128->1 [1][128], bn(1), fc1 [42][128], fc1_b [128], fc2 [128], fc2_b [1].
constexpr int kResChannels = 128;
constexpr int kResBlocks = 10;
constexpr int kResValueHidden = 128;
constexpr int kResInPlanes = 3;
constexpr float kBnEps = 1e-5f;

struct ResLayout {
  size_t stem_w, stem_bn;
  size_t conv1_w[kResBlocks], bn1[kResBlocks], conv2_w[kResBlocks], bn2[kResBlocks];
  size_t pol_w, pol_bn, pol_fc, pol_fc_b;
  size_t val_w, val_bn, val_fc1, val_fc1_b, val_fc2, val_fc2_b;
  size_t total;
};

GZ_HD ResLayout res_layout() {
  ResLayout t{};
  const size_t C = kResChannels;
  size_t o = 0;
  t.stem_w = o; o += C * 9 * kResInPlanes;
  t.stem_bn = o; o += 4 * C;
  for (int k = 0; k < kResBlocks; ++k) {
    t.conv1_w[k] = o; o += C * 9 * C;
    t.bn1[k] = o; o += 4 * C;
    t.conv2_w[k] = o; o += C * 9 * C;
    t.bn2[k] = o; o += 4 * C;
  }
  t.pol_w = o; o += 2 * C;
  t.pol_bn = o; o += 4 * 2;
  t.pol_fc = o; o += 84 * 7;
  t.pol_fc_b = o; o += 7;
  t.val_w = o; o += C;
  t.val_bn = o; o += 4;
  t.val_fc1 = o; o += 42 * kResValueHidden;
  t.val_fc1_b = o; o += kResValueHidden;
  t.val_fc2 = o; o += kResValueHidden;
  t.val_fc2_b = o; o += 1;
  t.total = o;
  return t;
}

}  // namespace gz
