// CPU oracle for the graphzero_b200 hot path.
//
// TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the CPU
// baseline legs of bench.py load this library, as the checker and as the
// timed CPU baseline.  The graphzero_b200 product never links or calls it.
//
// It restates, in plain fp32 (or fp64) loops with a fixed summation order:
//   * the board graphs, node features and game rules;
//   * the GAT forward the reference names but never finished
//     (networks/gat/gat.cu:150-198 predict, 836-870 forward_gat_layer,
//     916-948 compute_output; forward_gat is declared at gat.cuh:103 and never
//     defined), in the standard form: Wh = X W, e_ij = LeakyReLU_0.2(a_self.Wh_i
//     + a_nbr.Wh_j) over CSR neighbours j of i, alpha = softmax_j, out_i =
//     ELU(sum_j alpha_ij Wh_j + b), heads of 8 x 32;
//   * the Connect4 ResNet forward (networks/resnet/resnet.cu:506-667) with BN in
//     inference form and a real residual add (the reference overwrites,
//     resnet.cu:588-591);
//   * the batched PUCT wave algorithm (selection score of
//     self_play/self_play.cu:720-736, sign flip per level of 738-758,
//     expansion of 698-718 with P taken from the policy as at 627-629).
//
// Parity with the reference itself is unpinned for the network and the search:
// the reference has no tests, no golden vectors and does not build.  The game
// rules are pinned against the reference's own rule functions compiled under
// oracle/_ref (recipe: oracle/Makefile, target ref).
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace {

struct Shape {
  int N, rows, cols, A, F, L, P, board_bytes;
};

Shape shape_of(int game) {
  switch (game) {
    case 0: return {9, 3, 3, 9, 4, 4, 1, 9};          // TicTacToe
    case 1: return {42, 6, 7, 7, 4, 6, 1, 42};        // Connect4
    case 2: return {64, 8, 8, 4672, 18, 8, 73, 66};   // Chess (geometry + encoding)
  }
  return {0, 0, 0, 0, 0, 0, 0, 0};
}

constexpr int H = 256, NH = 8, HD = 32, VH = 64;

// ---------------------------------------------------------------- graphs ----
void graph_of(int game, std::vector<int>& rp, std::vector<int>& col) {
  Shape s = shape_of(game);
  rp.assign(s.N + 1, 0);
  col.clear();
  for (int i = 0; i < s.N; ++i) {
    rp[i] = (int)col.size();
    int ri = i / s.cols, ci = i % s.cols;
    for (int j = 0; j < s.N; ++j) {
      int dr = std::abs(j / s.cols - ri), dc = std::abs(j % s.cols - ci);
      bool nb;
      if (game == 2) {
        // queen lines (rank, file, diagonals; chess.cu:955-982) + knight
        // (chess.cu:995-1002) + self
        nb = dr == 0 || dc == 0 || dr == dc || (dr == 1 && dc == 2) || (dr == 2 && dc == 1);
      } else {
        nb = dr <= 1 && dc <= 1;  // king neighbourhood incl. self
      }
      if (nb) col.push_back(j);
    }
  }
  rp[s.N] = (int)col.size();
}

// -------------------------------------------------------------- features ----
void features(int game, const int8_t* b, int side, int node, float* f) {
  if (game != 2) {
    int v = b[node];
    f[0] = (float)(v == 0);
    f[1] = (float)(v == side);
    f[2] = (float)(v == -side);
    f[3] = (float)(side == 1);
    return;
  }
  for (int k = 0; k < 18; ++k) f[k] = 0.f;
  int v = b[node];
  if (v > 0) f[v - 1] = 1.f;
  if (v < 0) f[5 - v] = 1.f;
  f[12] = (float)(side == 1);
  unsigned c = (uint8_t)b[64];
  for (int k = 0; k < 4; ++k) f[13 + k] = (float)((c >> k) & 1u);
  f[17] = (float)(b[65] == node);
}

// ---------------------------------------------------------- blob layouts ----
struct GatOff {
  size_t W[8], b[8], a[8], w_pi, b_pi, W_v1, b_v1, w_v2, b_v2, total;
};

GatOff gat_off(int game) {
  Shape s = shape_of(game);
  GatOff o{};
  size_t p = 0;
  for (int l = 0; l < s.L; ++l) {
    int fin = l ? H : s.F;
    o.W[l] = p; p += (size_t)fin * H;
    o.b[l] = p; p += H;
    o.a[l] = p; p += NH * 2 * HD;
  }
  o.w_pi = p; p += (size_t)H * s.P;
  o.b_pi = p; p += s.P;
  o.W_v1 = p; p += (size_t)H * VH;
  o.b_v1 = p; p += VH;
  o.w_v2 = p; p += VH;
  o.b_v2 = p; p += 1;
  o.total = p;
  return o;
}

template <class T> T elu(T x) { return x > T(0) ? x : std::expm1(x); }
template <class T> T lrelu(T x) { return x > T(0) ? x : T(0.2) * x; }

// ------------------------------------------------------------ GAT (one) ----
template <class T>
void gat_one(int game, const float* w, const GatOff& o, const std::vector<int>& rp, const std::vector<int>& col,
             const int8_t* board, int side, float* pi, float* v) {
  Shape s = shape_of(game);
  const int N = s.N;
  std::vector<T> X((size_t)N * H), Wh((size_t)N * H), out((size_t)N * H);
  std::vector<T> ss((size_t)N * NH), sn((size_t)N * NH);
  std::vector<float> f(32);
  int fin = s.F;
  for (int i = 0; i < N; ++i) {
    features(game, board, side, i, f.data());
    for (int k = 0; k < fin; ++k) X[(size_t)i * H + k] = (T)f[k];
  }
  for (int l = 0; l < s.L; ++l) {
    const float* W = w + o.W[l];
    const float* bias = w + o.b[l];
    const float* a = w + o.a[l];
    // Wh = X W  (k ascending)
    for (int i = 0; i < N; ++i) {
      T* y = &Wh[(size_t)i * H];
      for (int c = 0; c < H; ++c) y[c] = T(0);
      for (int k = 0; k < fin; ++k) {
        T x = X[(size_t)i * H + k];
        const float* wr = W + (size_t)k * H;
        for (int c = 0; c < H; ++c) y[c] += x * (T)wr[c];
      }
    }
    // per-head scores
    for (int i = 0; i < N; ++i)
      for (int h = 0; h < NH; ++h) {
        T s0 = 0, s1 = 0;
        for (int d = 0; d < HD; ++d) {
          T x = Wh[(size_t)i * H + h * HD + d];
          s0 += (T)a[(h * 2 + 0) * HD + d] * x;
          s1 += (T)a[(h * 2 + 1) * HD + d] * x;
        }
        ss[i * NH + h] = s0;
        sn[i * NH + h] = s1;
      }
    // segment softmax + aggregation
    for (int i = 0; i < N; ++i) {
      T* y = &out[(size_t)i * H];
      for (int h = 0; h < NH; ++h) {
        T m = -INFINITY;
        for (int e = rp[i]; e < rp[i + 1]; ++e) m = std::max(m, lrelu<T>(ss[i * NH + h] + sn[col[e] * NH + h]));
        T z = 0;
        for (int e = rp[i]; e < rp[i + 1]; ++e) z += std::exp(lrelu<T>(ss[i * NH + h] + sn[col[e] * NH + h]) - m);
        for (int d = 0; d < HD; ++d) y[h * HD + d] = T(0);
        for (int e = rp[i]; e < rp[i + 1]; ++e) {
          int j = col[e];
          T al = std::exp(lrelu<T>(ss[i * NH + h] + sn[j * NH + h]) - m) / z;
          for (int d = 0; d < HD; ++d) y[h * HD + d] += al * Wh[(size_t)j * H + h * HD + d];
        }
      }
      for (int c = 0; c < H; ++c) X[(size_t)i * H + c] = elu<T>(y[c] + (T)bias[c]);
    }
    fin = H;
  }
  // value head: mean-pool -> 256x64 ReLU -> 64x1 -> tanh
  std::vector<T> g(H, T(0)), z(VH);
  for (int i = 0; i < N; ++i)
    for (int c = 0; c < H; ++c) g[c] += X[(size_t)i * H + c];
  for (int c = 0; c < H; ++c) g[c] /= (T)N;
  for (int u = 0; u < VH; ++u) {
    T acc = (T)w[o.b_v1 + u];
    for (int c = 0; c < H; ++c) acc += g[c] * (T)w[o.W_v1 + (size_t)c * VH + u];
    z[u] = acc > T(0) ? acc : T(0);
  }
  T vv = (T)w[o.b_v2];
  for (int u = 0; u < VH; ++u) vv += z[u] * (T)w[o.w_v2 + u];
  *v = (float)std::tanh(vv);
  // policy logits
  std::vector<T> logit(s.A);
  if (game == 0) {  // per-node 256 -> 1
    for (int i = 0; i < N; ++i) {
      T acc = (T)w[o.b_pi];
      for (int c = 0; c < H; ++c) acc += X[(size_t)i * H + c] * (T)w[o.w_pi + c];
      logit[i] = acc;
    }
  } else if (game == 1) {  // column mean-pool (6 rows) -> 256 -> 1
    for (int cc = 0; cc < 7; ++cc) {
      std::vector<T> m(H, T(0));
      for (int r = 0; r < 6; ++r)
        for (int c = 0; c < H; ++c) m[c] += X[(size_t)(r * 7 + cc) * H + c];
      T acc = (T)w[o.b_pi];
      for (int c = 0; c < H; ++c) acc += (m[c] / T(6)) * (T)w[o.w_pi + c];
      logit[cc] = acc;
    }
  } else {  // per-node 256 -> 73, index = square * 73 + type
    for (int i = 0; i < N; ++i)
      for (int t = 0; t < 73; ++t) {
        T acc = (T)w[o.b_pi + t];
        for (int c = 0; c < H; ++c) acc += X[(size_t)i * H + c] * (T)w[o.w_pi + (size_t)c * 73 + t];
        logit[i * 73 + t] = acc;
      }
  }
  T mx = -INFINITY;
  for (int a = 0; a < s.A; ++a) mx = std::max(mx, logit[a]);
  T zs = 0;
  for (int a = 0; a < s.A; ++a) zs += std::exp(logit[a] - mx);
  for (int a = 0; a < s.A; ++a) pi[a] = (float)(std::exp(logit[a] - mx) / zs);
}

// --------------------------------------------------------- ResNet (one) ----
struct ResOff {
  size_t stem_w, stem_bn, c1[10], b1[10], c2[10], b2[10];
  size_t pol_w, pol_bn, pol_fc, pol_fc_b, val_w, val_bn, val_fc1, val_fc1_b, val_fc2, val_fc2_b, total;
};

ResOff res_off() {
  ResOff o{};
  const size_t C = 128;
  size_t p = 0;
  o.stem_w = p; p += C * 9 * 3;
  o.stem_bn = p; p += 4 * C;
  for (int k = 0; k < 10; ++k) {
    o.c1[k] = p; p += C * 9 * C;
    o.b1[k] = p; p += 4 * C;
    o.c2[k] = p; p += C * 9 * C;
    o.b2[k] = p; p += 4 * C;
  }
  o.pol_w = p; p += 2 * C;
  o.pol_bn = p; p += 8;
  o.pol_fc = p; p += 84 * 7;
  o.pol_fc_b = p; p += 7;
  o.val_w = p; p += C;
  o.val_bn = p; p += 4;
  o.val_fc1 = p; p += 42 * 128;
  o.val_fc1_b = p; p += 128;
  o.val_fc2 = p; p += 128;
  o.val_fc2_b = p; p += 1;
  o.total = p;
  return o;
}

// y = gamma (x - mean) / sqrt(var + eps) + beta
template <class T> T bn(const float* p, int C, int c, T x) {
  T inv = T(1) / std::sqrt((T)p[3 * C + c] + (T)1e-5);
  return (T)p[c] * (x - (T)p[2 * C + c]) * inv + (T)p[C + c];
}

// 3x3 same-padding conv on a 6x7 board, activations [pos][C].
template <class T>
void conv3(const float* w, int cin, const std::vector<T>& x, std::vector<T>& y) {
  const int C = 128;
  y.assign((size_t)42 * C, T(0));
  for (int r = 0; r < 6; ++r)
    for (int c = 0; c < 7; ++c)
      for (int co = 0; co < C; ++co) {
        T acc = 0;
        for (int ky = 0; ky < 3; ++ky)
          for (int kx = 0; kx < 3; ++kx) {
            int rr = r + ky - 1, cc = c + kx - 1;
            if (rr < 0 || rr >= 6 || cc < 0 || cc >= 7) continue;
            const float* wr = w + (((size_t)co * 3 + ky) * 3 + kx) * cin;
            const T* xr = &x[(size_t)(rr * 7 + cc) * cin];
            for (int ci = 0; ci < cin; ++ci) acc += (T)wr[ci] * xr[ci];
          }
        y[(size_t)(r * 7 + c) * C + co] = acc;
      }
}

template <class T>
void res_one(const float* w, const ResOff& o, const int8_t* board, int side, float* pi, float* v) {
  const int C = 128;
  std::vector<T> x((size_t)42 * 3), a, t, u;
  for (int p = 0; p < 42; ++p) {
    x[p * 3 + 0] = (T)(board[p] == side);
    x[p * 3 + 1] = (T)(board[p] == -side);
    x[p * 3 + 2] = (T)(side == 1);
  }
  conv3<T>(w + o.stem_w, 3, x, t);
  a.resize(t.size());
  for (int p = 0; p < 42; ++p)
    for (int c = 0; c < C; ++c) a[p * C + c] = std::max(T(0), bn<T>(w + o.stem_bn, C, c, t[p * C + c]));
  for (int k = 0; k < 10; ++k) {
    conv3<T>(w + o.c1[k], C, a, t);
    for (int p = 0; p < 42; ++p)
      for (int c = 0; c < C; ++c) t[p * C + c] = std::max(T(0), bn<T>(w + o.b1[k], C, c, t[p * C + c]));
    conv3<T>(w + o.c2[k], C, t, u);
    for (int p = 0; p < 42; ++p)
      for (int c = 0; c < C; ++c) a[p * C + c] = std::max(T(0), bn<T>(w + o.b2[k], C, c, u[p * C + c]) + a[p * C + c]);
  }
  // policy: 1x1 conv -> 2 ch, BN, flatten (c * 42 + pos), FC 84 -> 7, softmax
  T feat[84];
  for (int ch = 0; ch < 2; ++ch)
    for (int p = 0; p < 42; ++p) {
      T acc = 0;
      for (int c = 0; c < C; ++c) acc += (T)w[o.pol_w + ch * C + c] * a[p * C + c];
      feat[ch * 42 + p] = bn<T>(w + o.pol_bn, 2, ch, acc);
    }
  T logit[7], mx = -INFINITY;
  for (int j = 0; j < 7; ++j) {
    T acc = (T)w[o.pol_fc_b + j];
    for (int i = 0; i < 84; ++i) acc += feat[i] * (T)w[o.pol_fc + i * 7 + j];
    logit[j] = acc;
    mx = std::max(mx, acc);
  }
  T zs = 0;
  for (int j = 0; j < 7; ++j) zs += std::exp(logit[j] - mx);
  for (int j = 0; j < 7; ++j) pi[j] = (float)(std::exp(logit[j] - mx) / zs);
  // value: 1x1 conv -> 1 ch, BN, FC 42 -> 128, ReLU, FC 128 -> 1, tanh
  T vf[42];
  for (int p = 0; p < 42; ++p) {
    T acc = 0;
    for (int c = 0; c < C; ++c) acc += (T)w[o.val_w + c] * a[p * C + c];
    vf[p] = bn<T>(w + o.val_bn, 1, 0, acc);
  }
  T vv = (T)w[o.val_fc2_b];
  for (int j = 0; j < 128; ++j) {
    T acc = (T)w[o.val_fc1_b + j];
    for (int p = 0; p < 42; ++p) acc += vf[p] * (T)w[o.val_fc1 + p * 128 + j];
    vv += std::max(T(0), acc) * (T)w[o.val_fc2 + j];
  }
  *v = (float)std::tanh(vv);
}

template <class F>
void parallel_for(int n, int nthreads, F fn) {
  if (nthreads <= 0) nthreads = (int)std::max(1u, std::thread::hardware_concurrency());
  nthreads = std::min(nthreads, std::max(1, n));
  if (nthreads == 1) {
    for (int i = 0; i < n; ++i) fn(i);
    return;
  }
  std::vector<std::thread> th;
  for (int t = 0; t < nthreads; ++t)
    th.emplace_back([=]() {
      for (int i = t; i < n; i += nthreads) fn(i);
    });
  for (auto& x : th) x.join();
}

// ----------------------------------------------------------------- rules ----
// Connect4 / TicTacToe rules restated from games/connect4/connect4.cu:22-93 and
// games/tictactoe/tictactoe.cu:24-72.
int apply_move(int game, int8_t* b, int a, int p) {
  if (game == 1) {
    for (int r = 5; r >= 0; --r)  // lowest empty row (connect4.cu:26-31)
      if (b[r * 7 + a] == 0) { b[r * 7 + a] = (int8_t)p; return r * 7 + a; }
    return -1;
  }
  if (b[a] != 0) return -1;
  b[a] = (int8_t)p;
  return a;
}

bool legal(int game, const int8_t* b, int a) {
  return game == 1 ? b[a] == 0 : b[a] == 0;  // top cell / square empty
}

// Whole-board scan for four (Connect4, connect4.cu:42-80) or a line
// (TicTacToe, tictactoe.cu:36-55) of player p.
bool has_won(int game, const int8_t* b, int p) {
  if (game == 1) {
    for (int r = 0; r < 6; ++r)
      for (int c = 0; c < 7; ++c) {
        if (b[r * 7 + c] != p) continue;
        if (c <= 3 && b[r * 7 + c + 1] == p && b[r * 7 + c + 2] == p && b[r * 7 + c + 3] == p) return true;
        if (r <= 2 && b[(r + 1) * 7 + c] == p && b[(r + 2) * 7 + c] == p && b[(r + 3) * 7 + c] == p) return true;
        if (c <= 3 && r <= 2 && b[(r + 1) * 7 + c + 1] == p && b[(r + 2) * 7 + c + 2] == p && b[(r + 3) * 7 + c + 3] == p)
          return true;
        if (c <= 3 && r >= 3 && b[(r - 1) * 7 + c + 1] == p && b[(r - 2) * 7 + c + 2] == p && b[(r - 3) * 7 + c + 3] == p)
          return true;
      }
    return false;
  }
  static const int L[8][3] = {{0, 1, 2}, {3, 4, 5}, {6, 7, 8}, {0, 3, 6}, {1, 4, 7}, {2, 5, 8}, {0, 4, 8}, {2, 4, 6}};
  for (auto& l : L)
    if (b[l[0]] == p && b[l[1]] == p && b[l[2]] == p) return true;
  return false;
}

// 1 = `moved` has won, 2 = draw (no legal move), 0 = continues.
int outcome(int game, const int8_t* b, int moved) {
  if (has_won(game, b, moved)) return 1;
  int A = shape_of(game).A;
  for (int a = 0; a < A; ++a)
    if (legal(game, b, a)) return 0;
  return 2;
}

// ------------------------------------------------------------------ MCTS ----
struct OEdge {
  float P, W;
  int N, VL, child, action;
};
struct ONode {
  int n, vl, first_edge, n_edges, side, expanded, terminal;
  float term_value;
  int8_t board[64];
};
struct OTree {
  std::vector<ONode> nodes;
  std::vector<OEdge> edges;
  int root;
  std::vector<std::vector<int>> pnodes, pedges;  // per leaf slot
};
struct OMcts {
  int game, trees, leaves, vl_k, node_cap, edge_cap;
  float c_puct;
  std::vector<OTree> t;
};

int new_node(OTree& t, const int8_t* board, int side, int term, float tv) {
  ONode n{};
  n.side = side;
  n.terminal = term;
  n.term_value = tv;
  n.first_edge = -1;
  memcpy(n.board, board, 64);
  t.nodes.push_back(n);
  return (int)t.nodes.size() - 1;
}

void reset_tree(OMcts& m, OTree& t, const int8_t* board, int side) {
  t.nodes.clear();
  t.edges.clear();
  int8_t b[64] = {0};
  memcpy(b, board, (size_t)shape_of(m.game).N);
  t.root = new_node(t, b, side, 0, 0.f);
}

// PUCT over the children of s; lowest index wins ties (strict >).
int puct_pick(const OMcts& m, const OTree& t, int s) {
  const ONode& nd = t.nodes[s];
  int np = nd.n + m.vl_k * nd.vl;
  float sq = std::sqrt((float)np);
  int best = -1;
  float bu = -INFINITY;
  for (int k = 0; k < nd.n_edges; ++k) {
    const OEdge& e = t.edges[nd.first_edge + k];
    int ne = e.N + m.vl_k * e.VL;
    float q = ne > 0 ? (e.W - (float)(m.vl_k * e.VL)) / (float)ne : 0.0f;
    float u1 = m.c_puct * e.P;
    float u2 = u1 * sq;
    float u3 = u2 / (1.0f + (float)ne);
    float u = q + u3;
    if (u > bu) { bu = u; best = nd.first_edge + k; }
  }
  return best;
}

// ------------------------------------------------------ synthetic inputs ----
// Seeded Glorot weights, BN parameters and random legal positions: the same
// splitmix64 streams as the product's generator (one stream per blob, one
// per position index), so the same seed gives bit-identical data and the CPU
// baseline can build its inputs without the product library.  The reference
// seeds cuRAND with time(NULL) (networks/gat/gat.cu:769), so it has no
// reproducible generator to follow.
struct Mix {
  uint64_t s;
  explicit Mix(uint64_t seed) : s(seed) {}
  uint64_t next() {  // splitmix64 (Steele, Lea, Flood 2014)
    uint64_t z = (s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
  }
  float uniform() { return (float)(next() >> 40) * (1.0f / 16777216.0f); }
  uint32_t below(uint32_t n) { return (uint32_t)(((next() >> 32) * (uint64_t)n) >> 32); }
  float normal() {  // Box-Muller on u1 in (0, 1], u2 in [0, 1)
    double u1 = ((double)(next() >> 11) + 1.0) * (1.0 / 9007199254740992.0);
    double u2 = (double)(next() >> 11) * (1.0 / 9007199254740992.0);
    return (float)(std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2));
  }
};

uint64_t stream_seed(uint64_t seed, uint64_t stream) { return Mix(seed ^ (stream * 0xD1B54A32D192ED03ull)).next(); }

float bf16_nearest(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7F800000u) == 0x7F800000u) return x;
  u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
  memcpy(&x, &u, 4);
  return x;
}

struct Gen {
  Mix r;
  float bias_scale;
  bool bf16;
  float q(float v) const { return bf16 ? bf16_nearest(v) : v; }
  void glorot(float* w, size_t n, int fan_in, int fan_out) {
    float lim = std::sqrt(6.0f / (float)(fan_in + fan_out));
    for (size_t i = 0; i < n; ++i) w[i] = q((2.0f * r.uniform() - 1.0f) * lim);
  }
  void bias(float* w, size_t n) {
    for (size_t i = 0; i < n; ++i) w[i] = q(bias_scale == 0.0f ? 0.0f : (2.0f * r.uniform() - 1.0f) * bias_scale);
  }
  void bn(float* b, int C) {  // gamma ~ U(0.8, 1.2), beta, mean ~ N(0, 0.1), var ~ U(0.5, 1.5)
    for (int c = 0; c < C; ++c) b[c] = 0.8f + 0.4f * r.uniform();
    for (int c = 0; c < C; ++c) b[C + c] = 0.1f * r.normal();
    for (int c = 0; c < C; ++c) b[2 * C + c] = 0.1f * r.normal();
    for (int c = 0; c < C; ++c) b[3 * C + c] = 0.5f + r.uniform();
    for (int i = 0; i < 4 * C; ++i) b[i] = q(b[i]);
  }
};

}  // namespace

extern "C" {

// GAT weights (gat_off layout), Glorot-uniform, biases U(+-bias_scale).
int orc_synth_gat_weights(int game, uint64_t seed, float bias_scale, int bf16_exact, float* out) {
  if (game < 0 || game > 2 || !out) return -1;
  Shape s = shape_of(game);
  GatOff o = gat_off(game);
  Gen g{Mix(stream_seed(seed, 0x6A7)), bias_scale, bf16_exact != 0};
  for (int l = 0; l < s.L; ++l) {
    int fin = l ? H : s.F;
    g.glorot(out + o.W[l], (size_t)fin * H, fin, H);
    g.bias(out + o.b[l], H);
    g.glorot(out + o.a[l], NH * 2 * HD, 2 * HD, 1);
  }
  g.glorot(out + o.w_pi, (size_t)H * s.P, H, s.P);
  g.bias(out + o.b_pi, s.P);
  g.glorot(out + o.W_v1, (size_t)H * VH, H, VH);
  g.bias(out + o.b_v1, VH);
  g.glorot(out + o.w_v2, VH, VH, 1);
  g.bias(out + o.b_v2, 1);
  return 0;
}

// Connect4 ResNet weights (res_off layout).
int orc_synth_res_weights(uint64_t seed, int bf16_exact, float* out) {
  if (!out) return -1;
  ResOff o = res_off();
  const int C = 128;
  Gen g{Mix(stream_seed(seed, 0x5E5)), 0.0f, bf16_exact != 0};
  g.glorot(out + o.stem_w, (size_t)C * 9 * 3, 9 * 3, 9 * C);
  g.bn(out + o.stem_bn, C);
  for (int k = 0; k < 10; ++k) {
    g.glorot(out + o.c1[k], (size_t)C * 9 * C, 9 * C, 9 * C);
    g.bn(out + o.b1[k], C);
    g.glorot(out + o.c2[k], (size_t)C * 9 * C, 9 * C, 9 * C);
    g.bn(out + o.b2[k], C);
  }
  g.glorot(out + o.pol_w, 2 * C, C, 2);
  g.bn(out + o.pol_bn, 2);
  g.glorot(out + o.pol_fc, 84 * 7, 84, 7);
  g.bias(out + o.pol_fc_b, 7);
  g.glorot(out + o.val_w, C, C, 1);
  g.bn(out + o.val_bn, 1);
  g.glorot(out + o.val_fc1, 42 * 128, 42, 128);
  g.bias(out + o.val_fc1_b, 128);
  g.glorot(out + o.val_fc2, 128, 128, 1);
  g.bias(out + o.val_fc2_b, 1);
  return 0;
}

// Random legal TicTacToe / Connect4 positions first .. first + n - 1 of the
// stream `seed`: k ~ U{0..N-1} uniformly random legal moves from the empty
// board, stopping before a move that would end the game.
int orc_synth_positions(int game, uint64_t seed, uint64_t first, int n, int8_t* boards, int8_t* side) {
  if (game != 0 && game != 1) return -1;
  Shape s = shape_of(game);
  for (int i = 0; i < n; ++i) {
    int8_t* b = boards + (size_t)i * s.board_bytes;
    Mix r(stream_seed(seed, 0x9051 + first + (uint64_t)i));
    memset(b, 0, (size_t)s.board_bytes);
    int k = (int)r.below((uint32_t)(s.N - 1) + 1), sd = 1;
    for (int ply = 0; ply < k; ++ply) {
      int moves[9], m = 0;
      for (int a = 0; a < s.A; ++a)
        if (legal(game, b, a)) moves[m++] = a;
      if (m == 0) break;
      int a = moves[r.below((uint32_t)m)];
      int8_t trial[64];
      memcpy(trial, b, (size_t)s.N);
      apply_move(game, trial, a, sd);
      if (outcome(game, trial, sd) != 0) break;
      memcpy(b, trial, (size_t)s.N);
      sd = -sd;
    }
    side[i] = (int8_t)sd;
  }
  return 0;
}

int orc_shape(int game, int* out) {
  Shape s = shape_of(game);
  std::vector<int> rp, col;
  graph_of(game, rp, col);
  int v[9] = {s.N, s.rows, s.cols, s.A, s.F, s.L, s.P, s.board_bytes, (int)col.size()};
  memcpy(out, v, sizeof v);
  return s.N ? 0 : -1;
}

int orc_graph(int game, int* row_ptr, int* col) {
  std::vector<int> rp, c;
  graph_of(game, rp, c);
  memcpy(row_ptr, rp.data(), rp.size() * sizeof(int));
  memcpy(col, c.data(), c.size() * sizeof(int));
  return (int)c.size();
}

void orc_features(int game, const int8_t* board, int side, float* out) {
  Shape s = shape_of(game);
  for (int i = 0; i < s.N; ++i) features(game, board, side, i, out + (size_t)i * s.F);
}

size_t orc_gat_weight_count(int game) { return gat_off(game).total; }
size_t orc_res_weight_count() { return res_off().total; }

int orc_gat_forward(int game, const float* w, const int8_t* boards, const int8_t* side, int B, float* pi, float* v,
                    int nthreads, int f64) {
  Shape s = shape_of(game);
  if (!s.N || B < 0) return -1;
  GatOff o = gat_off(game);
  std::vector<int> rp, col;
  graph_of(game, rp, col);
  parallel_for(B, nthreads, [&](int b) {
    const int8_t* bd = boards + (size_t)b * s.board_bytes;
    if (f64) gat_one<double>(game, w, o, rp, col, bd, side[b], pi + (size_t)b * s.A, v + b);
    else gat_one<float>(game, w, o, rp, col, bd, side[b], pi + (size_t)b * s.A, v + b);
  });
  return 0;
}

int orc_resnet_forward(const float* w, const int8_t* boards, const int8_t* side, int B, float* pi, float* v,
                       int nthreads, int f64) {
  ResOff o = res_off();
  parallel_for(B, nthreads, [&](int b) {
    if (f64) res_one<double>(w, o, boards + (size_t)b * 42, side[b], pi + (size_t)b * 7, v + b);
    else res_one<float>(w, o, boards + (size_t)b * 42, side[b], pi + (size_t)b * 7, v + b);
  });
  return 0;
}

int orc_apply(int game, int8_t* board, int action, int player) { return apply_move(game, board, action, player); }
int orc_legal(int game, const int8_t* board, int action) { return legal(game, board, action) ? 1 : 0; }
int orc_has_won(int game, const int8_t* board, int player) { return has_won(game, board, player) ? 1 : 0; }
int orc_outcome(int game, const int8_t* board, int moved) { return outcome(game, board, moved); }

// --- batched PUCT waves ------------------------------------------------------
void* orc_mcts_create(int game, int trees, int leaves, float c_puct, int vl_k, int node_cap) {
  OMcts* m = new OMcts();
  m->game = game;
  m->trees = trees;
  m->leaves = leaves;
  m->c_puct = c_puct;
  m->vl_k = vl_k;
  m->node_cap = node_cap;
  m->edge_cap = node_cap * shape_of(game).A;
  m->t.resize(trees);
  for (auto& t : m->t) {
    t.pnodes.resize(leaves);
    t.pedges.resize(leaves);
  }
  return m;
}

void orc_mcts_destroy(void* h) { delete (OMcts*)h; }

void orc_mcts_set_roots(void* h, const int8_t* boards, const int8_t* side) {
  OMcts& m = *(OMcts*)h;
  int N = shape_of(m.game).N;
  for (int i = 0; i < m.trees; ++i) reset_tree(m, m.t[i], boards + (size_t)i * N, side[i]);
}

// One selection pass: `leaves` sequential descents per tree with virtual loss.
// Writes each leaf's board [trees*leaves][N], side and terminal flag.
int orc_mcts_select(void* h, int8_t* out_boards, int8_t* out_side, int8_t* out_terminal) {
  OMcts& m = *(OMcts*)h;
  int N = shape_of(m.game).N;
  for (int ti = 0; ti < m.trees; ++ti) {
    OTree& t = m.t[ti];
    for (int k = 0; k < m.leaves; ++k) {
      auto& pn = t.pnodes[k];
      auto& pe = t.pedges[k];
      pn.clear();
      pe.clear();
      int s = t.root;
      pn.push_back(s);
      while (t.nodes[s].expanded && !t.nodes[s].terminal) {
        int e = puct_pick(m, t, s);
        t.nodes[s].vl += 1;
        t.edges[e].VL += 1;
        if (t.edges[e].child < 0) {
          if ((int)t.nodes.size() >= m.node_cap) return -2;
          int8_t b[64];
          memcpy(b, t.nodes[s].board, 64);
          int mover = t.nodes[s].side;
          apply_move(m.game, b, t.edges[e].action, mover);
          int oc = outcome(m.game, b, mover);
          // value for the side to move at the new node: it lost if the mover won
          int c = new_node(t, b, -mover, oc != 0, oc == 1 ? -1.0f : 0.0f);
          t.edges[e].child = c;
        }
        pe.push_back(e);
        s = t.edges[e].child;
        pn.push_back(s);
      }
      t.nodes[s].vl += 1;
      size_t slot = (size_t)ti * m.leaves + k;
      memcpy(out_boards + slot * N, t.nodes[s].board, (size_t)N);
      out_side[slot] = (int8_t)t.nodes[s].side;
      out_terminal[slot] = (int8_t)t.nodes[s].terminal;
    }
  }
  return 0;
}

// Backup of one wave in leaf order, expanding first-visited leaves with the
// policy renormalised over legal moves.
int orc_mcts_backup(void* h, const float* pi, const float* value) {
  OMcts& m = *(OMcts*)h;
  int A = shape_of(m.game).A;
  for (int ti = 0; ti < m.trees; ++ti) {
    OTree& t = m.t[ti];
    for (int k = 0; k < m.leaves; ++k) {
      size_t slot = (size_t)ti * m.leaves + k;
      auto& pn = t.pnodes[k];
      auto& pe = t.pedges[k];
      int leaf = pn.back();
      float v;
      if (t.nodes[leaf].terminal) {
        v = t.nodes[leaf].term_value;
      } else {
        v = value[slot];
        if (!t.nodes[leaf].expanded) {
          const float* p = pi + slot * A;
          float sum = 0.0f;
          int cnt = 0;
          for (int a = 0; a < A; ++a)
            if (legal(m.game, t.nodes[leaf].board, a)) { sum += p[a]; ++cnt; }
          if ((int)t.edges.size() + cnt > m.edge_cap) return -2;
          t.nodes[leaf].first_edge = (int)t.edges.size();
          t.nodes[leaf].n_edges = cnt;
          for (int a = 0; a < A; ++a)
            if (legal(m.game, t.nodes[leaf].board, a)) {
              OEdge e{};
              e.P = p[a] / sum;
              e.child = -1;
              e.action = a;
              t.edges.push_back(e);
            }
          t.nodes[leaf].expanded = 1;
        }
      }
      t.nodes[leaf].n += 1;
      t.nodes[leaf].vl -= 1;
      float val = -v;
      for (int i = (int)pe.size() - 1; i >= 0; --i) {
        OEdge& e = t.edges[pe[i]];
        e.N += 1;
        e.W += val;
        e.VL -= 1;
        ONode& nd = t.nodes[pn[i]];
        nd.n += 1;
        nd.vl -= 1;
        val = -val;
      }
    }
  }
  return 0;
}

// Root visit counts per action [trees][A] and root Q ([trees][A], W/N).
void orc_mcts_root_stats(void* h, int32_t* visits, float* wsum) {
  OMcts& m = *(OMcts*)h;
  int A = shape_of(m.game).A;
  for (int ti = 0; ti < m.trees; ++ti) {
    OTree& t = m.t[ti];
    const ONode& r = t.nodes[t.root];
    for (int a = 0; a < A; ++a) {
      visits[(size_t)ti * A + a] = 0;
      if (wsum) wsum[(size_t)ti * A + a] = 0.f;
    }
    for (int k = 0; k < r.n_edges; ++k) {
      const OEdge& e = t.edges[r.first_edge + k];
      visits[(size_t)ti * A + e.action] = e.N;
      if (wsum) wsum[(size_t)ti * A + e.action] = e.W;
    }
  }
}

// Node / edge totals per tree (used to compare tree shapes).
void orc_mcts_tree_sizes(void* h, int32_t* nodes, int32_t* edges) {
  OMcts& m = *(OMcts*)h;
  for (int ti = 0; ti < m.trees; ++ti) {
    nodes[ti] = (int32_t)m.t[ti].nodes.size();
    edges[ti] = (int32_t)m.t[ti].edges.size();
  }
}

// Advance every root by actions[tree].  The searched child becomes the new
// root and keeps its subtree (the reference's mcts_update_with_move,
// mcts/mcts.cu:68-103) while the pool still has `reserve` free nodes;
// otherwise the pool restarts from the new position alone.  A game that ended
// restarts from the empty board with the first player to move; done[tree] = 1.
void orc_mcts_play(void* h, const int32_t* actions, int reserve, int8_t* done) {
  OMcts& m = *(OMcts*)h;
  for (int ti = 0; ti < m.trees; ++ti) {
    OTree& t = m.t[ti];
    ONode r = t.nodes[t.root];
    int child = -1;
    for (int k = 0; k < r.n_edges; ++k)
      if (t.edges[r.first_edge + k].action == actions[ti]) child = t.edges[r.first_edge + k].child;
    int8_t b[64];
    memcpy(b, r.board, 64);
    int mover = r.side;
    apply_move(m.game, b, actions[ti], mover);
    int oc = outcome(m.game, b, mover);
    done[ti] = (int8_t)(oc != 0);
    if (oc) {
      int8_t e[64] = {0};
      reset_tree(m, t, e, 1);
    } else if (child >= 0 && (int)t.nodes.size() + reserve <= m.node_cap) {
      t.root = child;
    } else {
      reset_tree(m, t, b, -mover);
    }
  }
}

}  // extern "C"
