// INeuralNet / IGame shim over the C ABI: the reference's vtables
// (networks/neural_network.h:16-27, games/game.cuh:12-28) filled with
// functions that call graphzero_b200, so the reference's self-play, arena and
// player code can bind to this library unchanged.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <string>
#include <vector>

#include "../../include/graphzero_b200.h"
#include "../../include/graphzero_b200_compat.h"
#include "gz_games.h"
#include "gz_internal.h"
#include "gz_synth.h"

using namespace gz;

namespace {

struct GameImpl {
  IGame base;  // first member: IGame* and GameImpl* convert
  int game;
};

int game_of(const IGame* self) { return ((const GameImpl*)self)->game; }

void to_i8(const int* b, int n, int8_t* out) {
  for (int i = 0; i < n; ++i) out[i] = (int8_t)b[i];
}

void g_init(IGame*) {}
void g_init_board(const IGame* self, int* board) { memset(board, 0, sizeof(int) * game_shape(game_of(self)).nodes); }
void g_board_size(const IGame* self, int* rows, int* cols) {
  GameShape s = game_shape(game_of(self));
  *rows = s.rows;
  *cols = s.cols;
}
int g_action_size(const IGame* self) { return game_shape(game_of(self)).actions; }

// connect4.cu:22-34 / tictactoe.cu:24-31: an illegal action leaves the board
// unchanged (the reference's drop loop simply finds no empty cell).
void g_next_state(const IGame* self, const int* board, int player, int action, int* next_board, int* next_player) {
  const int g = game_of(self);
  GameShape s = game_shape(g);
  int8_t b[64];
  to_i8(board, s.nodes, b);
  if (action >= 0 && action < s.actions && action_legal(g, b, action)) apply_action(g, b, action, player);
  for (int i = 0; i < s.nodes; ++i) next_board[i] = b[i];
  *next_player = -player;
}

void g_valid_moves(const IGame* self, const int* board, int, bool* valid) {
  const int g = game_of(self);
  GameShape s = game_shape(g);
  int8_t b[64];
  to_i8(board, s.nodes, b);
  for (int a = 0; a < s.actions; ++a) valid[a] = action_legal(g, b, a);
}

int g_game_ended(const IGame* self, const int* board, int player) {
  const int g = game_of(self);
  GameShape s = game_shape(g);
  int8_t b[64];
  to_i8(board, s.nodes, b);
  int r = 0;
  if (gz_game_ended(g, b, player, &r) != GZ_OK) return 0;
  return r == 2 ? 0 : r;  // draw: 0, as the reference's int return type yields
}

void g_canonical(const IGame* self, const int* board, int player, int* out) {
  GameShape s = game_shape(game_of(self));
  for (int i = 0; i < s.nodes; ++i) out[i] = board[i] * player;
}

float g_evaluate(const IGame* self, const int* board, int player) { return (float)g_game_ended(self, board, player); }

// Board symmetries with the matching policy permutation: Connect4 mirror
// (connect4.cu:102-121), TicTacToe dihedral group (tictactoe.cu:107-146).
void g_symmetries(const IGame* self, const int* board, const float* pi, int (*sym)[GZ_MAX_BOARD_SIZE],
                  float (*sym_pi)[GZ_MAX_BOARD_SIZE], int* num) {
  const int g = game_of(self);
  if (g == kConnect4) {
    *num = 2;
    for (int i = 0; i < 42; ++i) sym[0][i] = board[i];
    for (int a = 0; a < 7; ++a) sym_pi[0][a] = pi[a];
    for (int r = 0; r < 6; ++r)
      for (int c = 0; c < 7; ++c) sym[1][r * 7 + c] = board[r * 7 + (6 - c)];
    for (int a = 0; a < 7; ++a) sym_pi[1][a] = pi[6 - a];
    return;
  }
  *num = 8;
  for (int t = 0; t < 8; ++t)
    for (int r = 0; r < 3; ++r)
      for (int c = 0; c < 3; ++c) {
        int rr = r, cc = c;
        for (int k = 0; k < (t & 3); ++k) {  // rotate 90 degrees k times
          int nr = cc, nc = 2 - rr;
          rr = nr;
          cc = nc;
        }
        if (t >= 4) cc = 2 - cc;  // then mirror
        sym[t][rr * 3 + cc] = board[r * 3 + c];
        sym_pi[t][rr * 3 + cc] = pi[r * 3 + c];
      }
}

void g_string(const IGame* self, const int* board, char* str, int str_size) {
  GameShape s = game_shape(game_of(self));
  const char sym[3] = {'O', '.', 'X'};
  int pos = 0;
  for (int r = 0; r < s.rows && pos < str_size - 1; ++r) {
    for (int c = 0; c < s.cols && pos < str_size - 1; ++c) str[pos++] = sym[board[r * s.cols + c] + 1];
    if (pos < str_size - 1) str[pos++] = '\n';
  }
  if (str_size > 0) str[pos] = '\0';
}

void g_display(const IGame* self, const int* board) {
  char buf[128];
  g_string(self, board, buf, sizeof buf);
  printf("%s\n", buf);
}

IGame* make_game(int g) {
  GameImpl* gi = (GameImpl*)calloc(1, sizeof(GameImpl));
  if (!gi) return nullptr;
  gi->game = g;
  IGame& b = gi->base;
  b.init = g_init;
  b.get_init_board = g_init_board;
  b.get_board_size = g_board_size;
  b.get_action_size = g_action_size;
  b.get_next_state = g_next_state;
  b.get_valid_moves = g_valid_moves;
  b.get_game_ended = g_game_ended;
  b.get_canonical_form = g_canonical;
  b.evaluate = g_evaluate;
  b.get_symmetries = g_symmetries;
  b.string_representation = g_string;
  b.display = g_display;
  return &gi->base;
}

// ---------------------------------------------------------------- network --
struct NetImpl {
  INeuralNet base;  // first member
  gz_net* net;
  bool owned;
};

gz_net* net_of(INeuralNet* self) { return ((NetImpl*)self)->net; }

void n_init(INeuralNet*, const IGame*) {}

// TrainingExample (networks/neural_network.h:10-14: canonical board and
// policy as float arrays, value) -> the library's example record.
bool to_records(gz_net* net, const float* const* boards, const float* const* pis, const float* vs, int n,
                std::vector<gz_train_example>& out) {
  int32_t shape[9];
  if (gz_game_shape(gz::net_game(net), shape) != GZ_OK) return false;
  const int nodes = shape[0], actions = shape[3];
  out.assign((size_t)n, gz_train_example{});
  for (int i = 0; i < n; ++i) {
    for (int k = 0; k < nodes; ++k) out[(size_t)i].board[k] = (int32_t)boards[i][k];
    for (int k = 0; k < actions; ++k) out[(size_t)i].pi[k] = pis[i][k];
    out[(size_t)i].v = vs[i];
  }
  return true;
}

// INeuralNet::train (gat.cu:82-148): the reference's defaults (10 passes,
// batches of 64, Adam 1e-3), one line of losses per call as it prints them.
void n_train(INeuralNet* self, TrainingExample* ex, int n) {
  gz_net* net = net_of(self);
  if (!ex || n <= 0) return;
  std::vector<const float*> b((size_t)n), p((size_t)n);
  std::vector<float> v((size_t)n);
  for (int i = 0; i < n; ++i) {
    b[(size_t)i] = ex[i].board;
    p[(size_t)i] = ex[i].pi;
    v[(size_t)i] = ex[i].v;
  }
  std::vector<gz_train_example> rec;
  gz_train_config cfg;
  gz_train_config_default(&cfg);
  gz_train_stats st{};
  if (!to_records(net, b.data(), p.data(), v.data(), n, rec) ||
      gz_net_train(net, rec.data(), n, &cfg, nullptr, 0, 1, &st) != GZ_OK) {
    fprintf(stderr, "graphzero_b200: train failed: %s\n", gz_last_error());
    return;
  }
  printf("Average Policy Loss: %f, Average Value Loss: %f\n", st.policy_loss, st.value_loss);
}

void n_predict(INeuralNet* self, const float* board, float* pi, float* v) {
  if (gz_net_predict(net_of(self), board, pi, v) != GZ_OK)
    fprintf(stderr, "graphzero_b200: predict failed: %s\n", gz_last_error());
}

std::string join(const char* folder, const char* file) {
  std::string p = folder ? folder : "";
  if (!p.empty() && p.back() != '/') p += '/';
  return p + (file ? file : "");
}

void n_save(INeuralNet* self, const char* folder, const char* file) {
  if (gz_net_save_checkpoint(net_of(self), join(folder, file).c_str()) != GZ_OK)
    fprintf(stderr, "graphzero_b200: save_checkpoint failed: %s\n", gz_last_error());
}

void n_load(INeuralNet* self, const char* folder, const char* file) {
  if (gz_net_load_checkpoint(net_of(self), join(folder, file).c_str()) != GZ_OK)
    fprintf(stderr, "graphzero_b200: load_checkpoint failed: %s\n", gz_last_error());
}

void n_destroy(INeuralNet* self) {
  NetImpl* ni = (NetImpl*)self;
  if (ni->owned) gz_net_destroy(ni->net);
  free(ni);
}

// INeuralNet::train_distributed (gat.cu:381-543): device arrays of canonical
// boards [n][nodes], policies [n][actions] and values [n].  Like the
// reference, rank 0's examples are broadcast first; every rank then trains
// on its slice of each step with the gradients all-reduced (data parallel;
// the reference's layer split across ranks is not kept).
void n_train_distributed(INeuralNet* self, float* d_boards, float* d_pis, float* d_vs, int n, int rank, int world,
                         void* comm, void* stream) {
  gz_net* net = net_of(self);
  int32_t shape[9];
  if (n <= 0 || gz_game_shape(gz::net_game(net), shape) != GZ_OK) return;
  const int nodes = shape[0], actions = shape[3];
  std::vector<float> hb((size_t)n * nodes), hp((size_t)n * actions), hv((size_t)n);
  if (gz::nccl_broadcast_floats(comm, d_boards, hb.size(), 0, stream) != GZ_OK ||
      gz::nccl_broadcast_floats(comm, d_pis, hp.size(), 0, stream) != GZ_OK ||
      gz::nccl_broadcast_floats(comm, d_vs, hv.size(), 0, stream) != GZ_OK ||
      cudaMemcpyAsync(hb.data(), d_boards, hb.size() * 4, cudaMemcpyDeviceToHost, (cudaStream_t)stream) ||
      cudaMemcpyAsync(hp.data(), d_pis, hp.size() * 4, cudaMemcpyDeviceToHost, (cudaStream_t)stream) ||
      cudaMemcpyAsync(hv.data(), d_vs, hv.size() * 4, cudaMemcpyDeviceToHost, (cudaStream_t)stream) ||
      cudaStreamSynchronize((cudaStream_t)stream)) {
    fprintf(stderr, "graphzero_b200: train_distributed: example broadcast failed: %s\n", gz_last_error());
    return;
  }
  std::vector<const float*> b((size_t)n), p((size_t)n);
  for (int i = 0; i < n; ++i) {
    b[(size_t)i] = hb.data() + (size_t)i * nodes;
    p[(size_t)i] = hp.data() + (size_t)i * actions;
  }
  std::vector<gz_train_example> rec;
  gz_train_config cfg;
  gz_train_config_default(&cfg);
  gz_train_stats st{};
  if (!to_records(net, b.data(), p.data(), hv.data(), n, rec) ||
      gz_net_train(net, rec.data(), n, &cfg, comm, rank, world, &st) != GZ_OK) {
    fprintf(stderr, "graphzero_b200: train_distributed failed: %s\n", gz_last_error());
    return;
  }
  if (rank == 0) printf("Average Policy Loss: %f, Average Value Loss: %f\n", st.policy_loss, st.value_loss);
}

void n_broadcast(INeuralNet* self, int, int, void* comm, void* stream) {
  if (gz_net_broadcast(net_of(self), comm, 0, stream) != GZ_OK)
    fprintf(stderr, "graphzero_b200: broadcast_weights failed: %s\n", gz_last_error());
}

INeuralNet* wrap(gz_net* net, bool owned) {
  NetImpl* ni = (NetImpl*)calloc(1, sizeof(NetImpl));
  if (!ni) return nullptr;
  ni->net = net;
  ni->owned = owned;
  INeuralNet& b = ni->base;
  b.impl = ni;
  b.init = n_init;
  b.train = n_train;
  b.predict = n_predict;
  b.save_checkpoint = n_save;
  b.load_checkpoint = n_load;
  b.destroy = n_destroy;
  b.train_distributed = n_train_distributed;
  b.broadcast_weights = n_broadcast;
  return &ni->base;
}

}  // namespace

extern "C" {

IGame* gz_create_connect4_game(void) { return make_game(kConnect4); }
IGame* gz_create_tictactoe_game(void) { return make_game(kTicTacToe); }
void gz_game_free(IGame* game) { free(game); }

INeuralNet* gz_create_neural_net(const char* net_type, const IGame* game, int device) {
  if (!net_type || !game) return nullptr;
  const int g = game_of(game);
  gz_net_config cfg{};
  cfg.game = g;
  cfg.precision = GZ_PREC_AUTO;
  cfg.max_batch = 1;
  if (strcmp(net_type, "gat") == 0) cfg.kind = GZ_NET_GAT;
  else if (strcmp(net_type, "resnet") == 0) cfg.kind = GZ_NET_RESNET;
  else return nullptr;
  gz_net* net = nullptr;
  if (gz_net_create(&cfg, device, &net) != GZ_OK) return nullptr;
  std::vector<float> w(gz_net_weight_count(net));
  WeightOpts o;
  if (cfg.kind == GZ_NET_GAT) make_gat_weights(g, 0x6A5A, o, w.data());
  else make_resnet_weights(0x6A5A, o, w.data());
  if (gz_net_load_weights(net, w.data(), w.size()) != GZ_OK) {
    gz_net_destroy(net);
    return nullptr;
  }
  INeuralNet* nn = wrap(net, true);
  if (!nn) gz_net_destroy(net);
  return nn;
}

gz_net* gz_shim_net(INeuralNet* nn) { return nn ? net_of(nn) : nullptr; }
INeuralNet* gz_shim_make_ineuralnet(gz_net* net) { return net ? wrap(net, false) : nullptr; }

}  // extern "C"
