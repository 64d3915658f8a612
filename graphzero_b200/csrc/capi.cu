// C ABI implementation: handles, argument checks, status codes, the
// host-buffer and single-position compatibility calls, NCCL weight broadcast,
// and the batched search driver.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <mutex>
#include <thread>
#include <vector>

#include "../../include/graphzero_b200.h"
#include "gz_games.h"
#include "gz_internal.h"
#include "gz_mcts.h"
#include "gz_sm100.h"
#include "gz_synth.h"
#include "gz_chess.h"
#include "gz_train.h"

using namespace gz;

namespace {

thread_local char g_err[512] = "";

gz_status fail(gz_status s, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
  return s;
}

}  // namespace

gz_status gz::set_last_error(gz_status s, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
  return s;
}

gz_status gz::forward_error_status(int err, const char* who) {
  if (!err) return GZ_OK;
  if (err == 2) return set_last_error(GZ_ERR_CUDA, "%s: dynamic shared memory base not 1024-byte aligned", who);
  return set_last_error(GZ_ERR_TIMEOUT, "%s: a bounded wait inside the kernel gave up (outputs of that launch are invalid)",
                        who);
}

namespace {

#define GZ_CUDA(call)                                                                                  \
  do {                                                                                                 \
    cudaError_t e_ = (call);                                                                           \
    if (e_ != cudaSuccess) return fail(GZ_ERR_CUDA, "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                                       __FILE__, __LINE__);                                           \
  } while (0)

// Restores the caller's current device on scope exit.
struct DeviceGuard {
  int prev = -1;
  bool ok = false;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) == cudaSuccess && cudaSetDevice(dev) == cudaSuccess) ok = true;
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

#define GZ_DEVICE(dev)                                                                      \
  DeviceGuard guard_((dev));                                                                \
  if (!guard_.ok) return fail(GZ_ERR_CUDA, "cannot select CUDA device %d", (int)(dev));

bool valid_game(int g) { return g == kTicTacToe || g == kConnect4 || g == kChess; }

// ---- NCCL, resolved at run time so the library has no link-time NCCL
// dependency (and shares the NCCL already loaded by the host process). ----
struct Nccl {
  void* h = nullptr;
  ncclResult_t (*getUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*commInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*allReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*errorString)(ncclResult_t) = nullptr;
};

Nccl* nccl() {
  static Nccl n;
  static std::once_flag once;
  std::call_once(once, [] {
    const char* names[] = {"libnccl.so.2", "libnccl.so"};
    for (const char* nm : names)
      if ((n.h = dlopen(nm, RTLD_NOW | RTLD_LOCAL))) break;
    if (!n.h) return;
    n.getUniqueId = (decltype(n.getUniqueId))dlsym(n.h, "ncclGetUniqueId");
    n.commInitRank = (decltype(n.commInitRank))dlsym(n.h, "ncclCommInitRank");
    n.commDestroy = (decltype(n.commDestroy))dlsym(n.h, "ncclCommDestroy");
    n.broadcast = (decltype(n.broadcast))dlsym(n.h, "ncclBroadcast");
    n.allReduce = (decltype(n.allReduce))dlsym(n.h, "ncclAllReduce");
    n.errorString = (decltype(n.errorString))dlsym(n.h, "ncclGetErrorString");
  });
  if (!n.h || !n.getUniqueId || !n.commInitRank || !n.commDestroy || !n.broadcast) return nullptr;
  return &n;
}

}  // namespace

struct gz_net {
  int game, kind, precision, device, max_batch;
  size_t weight_count;
  float* d_weights = nullptr;  // fp32 blob (source of truth on the device)
  int* d_csr = nullptr;        // row_ptr + col
  void* d_tc = nullptr;        // tensor-core packed weights (bf16 / fp16 path)
  size_t tc_bytes = 0;
  int* d_err = nullptr;        // sticky device error word of the forward kernels
  // host-call staging
  int8_t *h_in = nullptr, *d_in = nullptr;
  float *h_out = nullptr, *d_out = nullptr;
  cudaStream_t stream = nullptr;
  // host calls: a copy stream beside `stream`, and per half of a split call
  // the events "inputs copied", "forward done", "outputs copied"
  cudaStream_t copy_stream = nullptr;
  cudaEvent_t ev_in[4] = {}, ev_fwd[4] = {}, ev_out[4] = {};  // per piece of a host call
  gz::train::State* tr = nullptr;  // training state, created by the first training call
};

struct gz_mcts {
  MctsDev d{};
  int device;
  std::vector<void*> allocs;
  float *d_pi = nullptr, *d_v = nullptr;
  int32_t* d_tmp = nullptr;
};

struct gz_selfplay {
  SelfPlayDev s{};
  gz_mcts* m = nullptr;
  int device = 0;
  std::vector<void*> allocs;
  int32_t* d_actions = nullptr;
  int* d_counts = nullptr;  // out_count, games_done, overflow (contiguous)
};

namespace {

// GZ_PREC_AUTO resolved at creation: the fp32 SIMT kernel where no
// tensor-core kernel exists (TicTacToe), else the tensor-core kernel with
// fp16 operands (kAutoFp16).
int resolve_precision(int game, int kind, int precision) {
  if (precision != GZ_PREC_AUTO) return precision;
  if (kind == GZ_NET_GAT && (game == kTicTacToe || gat_tc_packed_bytes(game) == 0)) return GZ_PREC_FP32;
  return kAutoFp16 ? GZ_PREC_FP16 : GZ_PREC_BF16;
}

bool use_tensor_cores(const gz_net* n) {
  return n->kind == GZ_NET_GAT && (n->precision == GZ_PREC_BF16 || n->precision == GZ_PREC_FP16);
}

gz_status prepare_weights(gz_net* n, cudaStream_t s) {
  if (n->kind == GZ_NET_RESNET) {
    GZ_CUDA(launch_resnet_tc_pack(n->precision == GZ_PREC_FP16, n->d_weights, n->d_tc, s));
  } else if (n->kind == GZ_NET_GAT && use_tensor_cores(n)) {
    GZ_CUDA(launch_gat_tc_pack(n->game, n->precision == GZ_PREC_FP16, n->d_weights, n->d_tc, s));
  }
  return GZ_OK;
}

gz_status run_forward(gz_net* n, const int8_t* boards, const int8_t* side, int count, float* pi, float* v,
                      cudaStream_t s) {
  if (n->kind == GZ_NET_GAT) {
    if (use_tensor_cores(n))
      GZ_CUDA(launch_gat_tc(n->game, n->precision == GZ_PREC_FP16, n->d_tc, n->d_weights, boards, side, count, pi, v,
                            n->d_err, s));
    else
      GZ_CUDA(launch_gat_simt(n->game, n->d_weights, n->d_csr, boards, side, count, pi, v, s));
    return GZ_OK;
  }
  GZ_CUDA(launch_resnet_tc(n->precision == GZ_PREC_FP16, n->d_tc, n->d_weights, boards, side, count, pi, v, n->d_err, s));
  return GZ_OK;
}

}  // namespace

extern "C" {

const char* gz_status_string(gz_status s) {
  switch (s) {
    case GZ_OK: return "ok";
    case GZ_ERR_INVALID_ARG: return "invalid argument";
    case GZ_ERR_CUDA: return "CUDA error";
    case GZ_ERR_NCCL: return "NCCL error";
    case GZ_ERR_TIMEOUT: return "timeout";
    case GZ_ERR_IO: return "I/O error";
    case GZ_ERR_CAPACITY: return "capacity exceeded";
    case GZ_ERR_UNSUPPORTED: return "unsupported";
  }
  return "unknown status";
}

const char* gz_last_error(void) { return g_err; }
const char* gz_version(void) { return "graphzero_b200 0.1 (sm_100a)"; }

gz_status gz_game_shape(int game, int32_t out[9]) {
  if (!valid_game(game) || !out) return fail(GZ_ERR_INVALID_ARG, "bad game %d", game);
  GameShape s = game_shape(game);
  int32_t v[9] = {s.nodes, s.rows, s.cols, s.actions, s.features, s.layers, s.policy_out, s.board_bytes, s.nnz};
  memcpy(out, v, sizeof v);
  return GZ_OK;
}

gz_status gz_game_graph(int game, int32_t* row_ptr, int32_t* col) {
  if (!valid_game(game) || !row_ptr || !col) return fail(GZ_ERR_INVALID_ARG, "bad arguments");
  build_graph_csr(game, row_ptr, col);
  return GZ_OK;
}

gz_status gz_game_next_state(int game, const int8_t* board, int player, int action, int8_t* next_board,
                             int* next_player) {
  if ((game != kTicTacToe && game != kConnect4) || !board || !next_board || !next_player || (player != 1 && player != -1))
    return fail(GZ_ERR_INVALID_ARG, "bad arguments");
  GameShape s = game_shape(game);
  if (action < 0 || action >= s.actions || !action_legal(game, board, action))
    return fail(GZ_ERR_INVALID_ARG, "illegal action %d", action);
  memmove(next_board, board, (size_t)s.nodes);
  apply_action(game, next_board, action, player);
  *next_player = -player;
  return GZ_OK;
}

gz_status gz_game_valid_moves(int game, const int8_t* board, uint8_t* valid) {
  if ((game != kTicTacToe && game != kConnect4) || !board || !valid) return fail(GZ_ERR_INVALID_ARG, "bad arguments");
  GameShape s = game_shape(game);
  for (int a = 0; a < s.actions; ++a) valid[a] = action_legal(game, board, a) ? 1 : 0;
  return GZ_OK;
}

gz_status gz_game_ended(int game, const int8_t* board, int player, int* result) {
  if ((game != kTicTacToe && game != kConnect4) || !board || !result || (player != 1 && player != -1))
    return fail(GZ_ERR_INVALID_ARG, "bad arguments");
  GameShape s = game_shape(game);
  // A win is a line through some stone; check every stone of each player.
  int won = 0;
  for (int p = 1; p >= -1 && !won; p -= 2)
    for (int i = 0; i < s.nodes && !won; ++i)
      if (board[i] == p) {
        bool w = game == kConnect4 ? c4_win_through(board, i / 7, i % 7, p) : ttt_line_win(board, p);
        if (w) won = p;
      }
  if (won) {
    *result = won == player ? 1 : -1;
    return GZ_OK;
  }
  bool full = true;
  for (int a = 0; a < s.actions; ++a)
    if (action_legal(game, board, a)) full = false;
  *result = full ? 2 : 0;
  return GZ_OK;
}

size_t gz_weight_count(int game, int kind) {
  if (kind == GZ_NET_RESNET) return game == kConnect4 ? res_layout().total : 0;
  if (kind == GZ_NET_GAT && valid_game(game)) return gat_layout(game).total;
  return 0;
}

gz_status gz_synth_weights(int game, int kind, uint64_t seed, float bias_scale, int bf16_exact, float* out,
                           size_t n_floats) {
  size_t need = gz_weight_count(game, kind);
  if (!need || !out || n_floats != need) return fail(GZ_ERR_INVALID_ARG, "weight buffer must hold %zu floats", need);
  WeightOpts o;
  o.bias_scale = bias_scale;
  o.bf16_exact = bf16_exact != 0;
  if (kind == GZ_NET_GAT) make_gat_weights(game, seed, o, out);
  else make_resnet_weights(seed, o, out);
  return GZ_OK;
}

gz_status gz_synth_positions(int game, uint64_t seed, uint64_t first, int n, int8_t* boards, int8_t* side) {
  if (!valid_game(game) || n < 0 || (n > 0 && (!boards || !side))) return fail(GZ_ERR_INVALID_ARG, "bad arguments");
  GameShape s = game_shape(game);
  if (game != kChess) {
    for (int i = 0; i < n; ++i)
      side[i] = (int8_t)make_position(game, seed, first + (uint64_t)i, boards + (size_t)i * s.board_bytes);
    return GZ_OK;
  }
  // Chess playouts cost ~0.3 ms each: positions are independent (each is a
  // function of its stream index), so host threads split the range.
  auto run = [&](int lo, int hi) {
    for (int i = lo; i < hi; ++i)
      side[i] = (int8_t)chess::make_position(seed, first + (uint64_t)i, boards + (size_t)i * s.board_bytes);
  };
  int threads = (int)std::thread::hardware_concurrency();
  threads = threads < 1 ? 1 : threads > 64 ? 64 : threads;
  if (n < 64 || threads == 1) {
    run(0, n);
    return GZ_OK;
  }
  std::vector<std::thread> pool;
  for (int t = 0; t < threads; ++t) pool.emplace_back(run, (int)((int64_t)n * t / threads), (int)((int64_t)n * (t + 1) / threads));
  for (auto& th : pool) th.join();
  return GZ_OK;
}

gz_status gz_chess_legal_count(const int8_t* board, int side, int* count) {
  if (!board || !count || (side != 1 && side != -1)) return fail(GZ_ERR_INVALID_ARG, "bad arguments");
  chess::Pos p;
  chess::from_record(board, side, p);
  chess::Move ms[256];
  *count = chess::legal_moves(p, ms);
  return GZ_OK;
}

gz_status gz_chess_perft(const int8_t* board, int side, int depth, uint64_t* nodes) {
  if (!board || !nodes || (side != 1 && side != -1) || depth < 0 || depth > 6)
    return fail(GZ_ERR_INVALID_ARG, "bad arguments (depth 0..6)");
  chess::Pos p;
  chess::from_record(board, side, p);
  *nodes = chess::perft(p, depth);
  return GZ_OK;
}

gz_status gz_chess_legal_actions(const int8_t* board, int side, int16_t* actions, int* count) {
  if (!board || !actions || !count || (side != 1 && side != -1)) return fail(GZ_ERR_INVALID_ARG, "bad arguments");
  chess::Pos p;
  chess::from_record(board, side, p);
  chess::Move ms[256];
  const int c = chess::legal_moves(p, ms);
  for (int k = 0; k < c; ++k) actions[k] = (int16_t)chess::encode_action(ms[k]);
  *count = c;
  return GZ_OK;
}

gz_status gz_chess_valid_moves(const int8_t* board, int side, uint8_t* valid) {
  if (!board || !valid || (side != 1 && side != -1)) return fail(GZ_ERR_INVALID_ARG, "bad arguments");
  chess::Pos p;
  chess::from_record(board, side, p);
  chess::Move ms[256];
  const int c = chess::legal_moves(p, ms);
  memset(valid, 0, 64 * 73);
  for (int k = 0; k < c; ++k) valid[chess::encode_action(ms[k])] = 1;
  return GZ_OK;
}

gz_status gz_chess_next_state(const int8_t* board, int side, int action, int8_t* next_board, int* next_side) {
  if (!board || !next_board || !next_side || (side != 1 && side != -1)) return fail(GZ_ERR_INVALID_ARG, "bad arguments");
  chess::Pos p;
  chess::from_record(board, side, p);
  chess::Move m;
  if (!chess::find_action(p, action, &m)) return fail(GZ_ERR_INVALID_ARG, "illegal action %d", action);
  chess::apply(p, m);
  chess::to_record(p, next_board);
  *next_side = p.side;
  return GZ_OK;
}

gz_status gz_chess_ended(const int8_t* board, int side, int* result) {
  if (!board || !result || (side != 1 && side != -1)) return fail(GZ_ERR_INVALID_ARG, "bad arguments");
  chess::Pos p;
  chess::from_record(board, side, p);
  *result = chess::outcome(p);
  return GZ_OK;
}

gz_status gz_synth_positions_device(int game, uint64_t seed, uint64_t first, int n, int8_t* d_boards, int8_t* d_side,
                                    void* stream) {
  if (!valid_game(game) || n < 0 || (n > 0 && (!d_boards || !d_side))) return fail(GZ_ERR_INVALID_ARG, "bad arguments");
  GZ_CUDA(launch_synth_positions(game, seed, first, n, d_boards, d_side, (cudaStream_t)stream));
  return GZ_OK;
}

gz_status gz_chess_legal_actions_device(const int8_t* d_boards, const int8_t* d_side, int n, int16_t* d_actions,
                                        int32_t* d_counts, void* stream) {
  if (n < 0 || (n > 0 && (!d_boards || !d_side || !d_actions || !d_counts))) return fail(GZ_ERR_INVALID_ARG, "bad arguments");
  GZ_CUDA(launch_chess_legal(d_boards, d_side, n, d_actions, d_counts, (cudaStream_t)stream));
  return GZ_OK;
}

gz_status gz_net_create(const gz_net_config* cfg, int device, gz_net** out) {
  if (!cfg || !out) return fail(GZ_ERR_INVALID_ARG, "null argument");
  *out = nullptr;
  if (!valid_game(cfg->game)) return fail(GZ_ERR_INVALID_ARG, "bad game %d", cfg->game);
  if (cfg->kind != GZ_NET_GAT && cfg->kind != GZ_NET_RESNET) return fail(GZ_ERR_INVALID_ARG, "bad kind %d", cfg->kind);
  if (cfg->kind == GZ_NET_RESNET && cfg->game != kConnect4)
    return fail(GZ_ERR_UNSUPPORTED, "the ResNet tower is built for Connect4 only");
  if (cfg->kind == GZ_NET_RESNET && cfg->precision == GZ_PREC_FP32)
    return fail(GZ_ERR_UNSUPPORTED, "the ResNet tower runs on tensor cores (bf16 or fp16 operands)");
  if (cfg->precision < GZ_PREC_AUTO || cfg->precision > GZ_PREC_FP16) return fail(GZ_ERR_INVALID_ARG, "bad precision");
  if (cfg->max_batch < 0) return fail(GZ_ERR_INVALID_ARG, "bad max_batch");
  int ndev = 0;
  GZ_CUDA(cudaGetDeviceCount(&ndev));
  if (device < 0 || device >= ndev) return fail(GZ_ERR_INVALID_ARG, "device %d of %d", device, ndev);
  GZ_DEVICE(device);
  gz_net* n = new gz_net();
  n->game = cfg->game;
  n->kind = cfg->kind;
  n->precision = resolve_precision(cfg->game, cfg->kind, cfg->precision);
  n->device = device;
  n->max_batch = cfg->max_batch > 0 ? cfg->max_batch : 1;
  n->weight_count = gz_weight_count(cfg->game, cfg->kind);
  GameShape s = game_shape(cfg->game);
  gz_status st = GZ_OK;
  auto chk = [&](cudaError_t e, const char* what) {
    if (e != cudaSuccess && st == GZ_OK) st = fail(GZ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  };
  chk(cudaMalloc(&n->d_weights, n->weight_count * sizeof(float)), "cudaMalloc weights");
  chk(cudaMemset(n->d_weights, 0, n->weight_count * sizeof(float)), "cudaMemset weights");
  std::vector<int> csr(s.nodes + 1 + s.nnz);
  build_graph_csr(cfg->game, csr.data(), csr.data() + s.nodes + 1);
  chk(cudaMalloc(&n->d_csr, csr.size() * sizeof(int)), "cudaMalloc csr");
  chk(cudaMalloc(&n->d_err, sizeof(int)), "cudaMalloc err");
  chk(cudaMemset(n->d_err, 0, sizeof(int)), "cudaMemset err");
  chk(cudaMemcpy(n->d_csr, csr.data(), csr.size() * sizeof(int), cudaMemcpyHostToDevice), "copy csr");
  if (cfg->kind == GZ_NET_RESNET) {
    n->tc_bytes = resnet_tc_packed_bytes();
    chk(cudaMalloc(&n->d_tc, n->tc_bytes), "cudaMalloc packed weights");
  } else if (use_tensor_cores(n)) {
    n->tc_bytes = gat_tc_packed_bytes(cfg->game);
    if (!n->tc_bytes && st == GZ_OK) st = fail(GZ_ERR_UNSUPPORTED, "no tensor-core kernel for game %d", cfg->game);
    else chk(cudaMalloc(&n->d_tc, n->tc_bytes), "cudaMalloc packed weights");
  }
  size_t in_bytes = (size_t)n->max_batch * (s.board_bytes + 1);
  size_t out_floats = (size_t)n->max_batch * (s.actions + 1);
  chk(cudaMallocHost(&n->h_in, in_bytes), "cudaMallocHost in");
  chk(cudaMalloc(&n->d_in, in_bytes), "cudaMalloc in");
  // + one word after the outputs: the error word, copied back with them
  chk(cudaMallocHost(&n->h_out, (out_floats + 1) * sizeof(float)), "cudaMallocHost out");
  chk(cudaMalloc(&n->d_out, out_floats * sizeof(float)), "cudaMalloc out");
  chk(cudaStreamCreateWithFlags(&n->stream, cudaStreamNonBlocking), "stream");
  chk(cudaStreamCreateWithFlags(&n->copy_stream, cudaStreamNonBlocking), "copy stream");
  for (int h = 0; h < 4; ++h) {
    chk(cudaEventCreateWithFlags(&n->ev_in[h], cudaEventDisableTiming), "event");
    chk(cudaEventCreateWithFlags(&n->ev_fwd[h], cudaEventDisableTiming), "event");
    chk(cudaEventCreateWithFlags(&n->ev_out[h], cudaEventDisableTiming), "event");
  }
  if (st == GZ_OK) {
    gz_status p = prepare_weights(n, n->stream);
    if (p != GZ_OK) st = p;
  }
  if (st == GZ_OK) chk(cudaStreamSynchronize(n->stream), "sync");
  if (st != GZ_OK) {
    gz_net_destroy(n);
    return st;
  }
  *out = n;
  return GZ_OK;
}

gz_status gz_net_destroy(gz_net* n) {
  if (!n) return GZ_OK;
  DeviceGuard g(n->device);
  if (n->stream) cudaStreamSynchronize(n->stream);
  if (n->copy_stream) cudaStreamSynchronize(n->copy_stream);
  if (n->tr) {
    gz::train::free_state(*n->tr);
    delete n->tr;
  }
  cudaFree(n->d_weights);
  cudaFree(n->d_csr);
  cudaFree(n->d_tc);
  cudaFree(n->d_err);
  cudaFreeHost(n->h_in);
  cudaFree(n->d_in);
  cudaFreeHost(n->h_out);
  cudaFree(n->d_out);
  if (n->stream) cudaStreamDestroy(n->stream);
  if (n->copy_stream) cudaStreamDestroy(n->copy_stream);
  for (int h = 0; h < 4; ++h) {
    if (n->ev_in[h]) cudaEventDestroy(n->ev_in[h]);
    if (n->ev_fwd[h]) cudaEventDestroy(n->ev_fwd[h]);
    if (n->ev_out[h]) cudaEventDestroy(n->ev_out[h]);
  }
  delete n;
  return GZ_OK;
}

size_t gz_net_weight_count(const gz_net* n) { return n ? n->weight_count : 0; }

const char* gz_net_kernel_name(const gz_net* n) {
  if (!n) return "";
  if (n->kind == GZ_NET_RESNET) return n->precision == GZ_PREC_FP16 ? "resnet_tc_fp16" : "resnet_tc_bf16";
  if (!use_tensor_cores(n)) return "gat_simt_fp32";
  return n->precision == GZ_PREC_FP16 ? "gat_tc_fp16" : "gat_tc_bf16";  // gat_tc_c4_kernel
}

gz_status gz_net_load_weights(gz_net* n, const float* blob, size_t count) {
  if (!n || !blob) return fail(GZ_ERR_INVALID_ARG, "null argument");
  if (count != n->weight_count) return fail(GZ_ERR_INVALID_ARG, "weight blob has %zu floats, expected %zu", count, n->weight_count);
  GZ_DEVICE(n->device);
  GZ_CUDA(cudaMemcpyAsync(n->d_weights, blob, count * sizeof(float), cudaMemcpyHostToDevice, n->stream));
  gz_status p = prepare_weights(n, n->stream);
  if (p != GZ_OK) return p;
  GZ_CUDA(cudaStreamSynchronize(n->stream));
  return GZ_OK;
}

gz_status gz_net_save_weights(const gz_net* n, float* blob, size_t count) {
  if (!n || !blob) return fail(GZ_ERR_INVALID_ARG, "null argument");
  if (count != n->weight_count) return fail(GZ_ERR_INVALID_ARG, "weight blob has %zu floats, expected %zu", count, n->weight_count);
  GZ_DEVICE(n->device);
  GZ_CUDA(cudaMemcpyAsync(blob, n->d_weights, count * sizeof(float), cudaMemcpyDeviceToHost, n->stream));
  GZ_CUDA(cudaStreamSynchronize(n->stream));
  return GZ_OK;
}

namespace {
uint64_t fnv1a(const void* data, size_t bytes) {
  const uint8_t* p = (const uint8_t*)data;
  uint64_t h = 1469598103934665603ull;
  for (size_t i = 0; i < bytes; ++i) h = (h ^ p[i]) * 1099511628211ull;
  return h;
}
struct CkptHeader {
  char magic[8];
  int32_t version, game, kind, reserved;
  uint64_t count;
};
}  // namespace

gz_status gz_net_save_checkpoint(const gz_net* n, const char* path) {
  if (!n || !path) return fail(GZ_ERR_INVALID_ARG, "null argument");
  std::vector<float> w(n->weight_count);
  gz_status st = gz_net_save_weights(n, w.data(), w.size());
  if (st != GZ_OK) return st;
  CkptHeader h{};
  memcpy(h.magic, "GZB200W1", 8);
  h.version = 1;
  h.game = n->game;
  h.kind = n->kind;
  h.count = w.size();
  uint64_t hash = fnv1a(w.data(), w.size() * sizeof(float));
  FILE* f = fopen(path, "wb");
  if (!f) return fail(GZ_ERR_IO, "cannot open %s for writing", path);
  bool ok = fwrite(&h, sizeof h, 1, f) == 1 && fwrite(w.data(), sizeof(float), w.size(), f) == w.size() &&
            fwrite(&hash, sizeof hash, 1, f) == 1;
  ok = (fclose(f) == 0) && ok;
  return ok ? GZ_OK : fail(GZ_ERR_IO, "short write to %s", path);
}

gz_status gz_net_load_checkpoint(gz_net* n, const char* path) {
  if (!n || !path) return fail(GZ_ERR_INVALID_ARG, "null argument");
  FILE* f = fopen(path, "rb");
  if (!f) return fail(GZ_ERR_IO, "cannot open %s", path);
  CkptHeader h{};
  std::vector<float> w;
  uint64_t hash = 0;
  gz_status st = GZ_OK;
  if (fread(&h, sizeof h, 1, f) != 1 || memcmp(h.magic, "GZB200W1", 8) != 0 || h.version != 1) {
    st = fail(GZ_ERR_IO, "%s: not a graphzero_b200 checkpoint", path);
  } else if (h.game != n->game || h.kind != n->kind || h.count != n->weight_count) {
    st = fail(GZ_ERR_IO, "%s: checkpoint for game %d kind %d (%llu weights) does not fit this net", path, h.game,
              h.kind, (unsigned long long)h.count);
  } else {
    w.resize(h.count);
    if (fread(w.data(), sizeof(float), w.size(), f) != w.size() || fread(&hash, sizeof hash, 1, f) != 1)
      st = fail(GZ_ERR_IO, "%s: truncated checkpoint", path);
    else if (hash != fnv1a(w.data(), w.size() * sizeof(float)))
      st = fail(GZ_ERR_IO, "%s: checksum mismatch", path);
  }
  fclose(f);
  if (st != GZ_OK) return st;
  return gz_net_load_weights(n, w.data(), w.size());
}

gz_status gz_net_predict_batch(gz_net* n, const int8_t* boards, const int8_t* side, int count, float* pi, float* v,
                               void* stream) {
  if (!n) return fail(GZ_ERR_INVALID_ARG, "null net");
  if (count < 0) return fail(GZ_ERR_INVALID_ARG, "negative batch");
  if (count == 0) return GZ_OK;
  if (!boards || !side || !pi || !v) return fail(GZ_ERR_INVALID_ARG, "null buffer");
  GZ_DEVICE(n->device);
  return run_forward(n, boards, side, count, pi, v, (cudaStream_t)stream);
}

// Turns a nonzero device error word into a status (and clears the word).
static gz_status forward_error(gz_net* n, int err) {
  if (!err) return GZ_OK;
  GZ_CUDA(cudaMemset(n->d_err, 0, sizeof(int)));
  return gz::forward_error_status(err, "forward kernel");
}

gz_status gz_net_check(gz_net* n) {
  if (!n) return fail(GZ_ERR_INVALID_ARG, "null net");
  GZ_DEVICE(n->device);
  int err = 0;
  GZ_CUDA(cudaMemcpy(&err, n->d_err, sizeof(int), cudaMemcpyDeviceToHost));
  return forward_error(n, err);
}

namespace {
// Page-locked host memory (cudaHostAlloc / cudaHostRegister): the copy
// engines read and write it directly.
bool page_locked(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeHost;
}
// The device-side address of page-locked host memory that is mapped into the
// device's address space (cudaHostAlloc'd memory is, with unified
// addressing), or null.
void* mapped_address(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return a.type == cudaMemoryTypeHost ? a.devicePointer : nullptr;
}
constexpr int kSplitMin = 1024;  // chess host calls at least this large run as overlapped pieces
constexpr int kPieces = 4;       // pieces of such a call (at most 4, the events per net)
}  // namespace

gz_status gz_net_predict_host(gz_net* n, const int8_t* boards, const int8_t* side, int count, float* pi, float* v) {
  if (!n) return fail(GZ_ERR_INVALID_ARG, "null net");
  if (count < 0 || count > n->max_batch) return fail(GZ_ERR_INVALID_ARG, "batch %d outside [0, %d]", count, n->max_batch);
  if (count == 0) return GZ_OK;
  if (!boards || !side || !pi || !v) return fail(GZ_ERR_INVALID_ARG, "null buffer");
  GZ_DEVICE(n->device);
  GameShape s = game_shape(n->game);
  const size_t bb = (size_t)count * s.board_bytes;
  int8_t* d_boards = n->d_in;
  int8_t* d_side = n->d_in + bb;
  float* d_pi = n->d_out;
  float* d_v = n->d_out + (size_t)count * s.actions;
  // the error word rides in the same stream as the outputs (no second round trip)
  int* h_err = (int*)(n->h_out + (size_t)n->max_batch * (s.actions + 1));

  // A large chess call runs in pieces: inputs on the copy stream, forward
  // passes on the compute stream, outputs back on the copy stream once each
  // piece's forward pass is done, so that one piece's transfers (and, for
  // pageable caller buffers, host copies) overlap the next piece's forward
  // pass.  The split points are multiples of 6, so every position keeps its
  // slot in the kernels' tiles (2 or 3 positions each) and the results are
  // the unsplit call's bit for bit.  Measured on B200 from page-locked
  // buffers, chess 8192 positions (153 MB of policy back to the host): 5.06
  // ms per call unsplit, 3.90 in two pieces, 3.35 in four.  Connect4 runs
  // unsplit: its outputs are small (GAT 4096: 381 µs per call unsplit, 383
  // in two pieces), and the ResNet kernel runs its tiles in pairs per CTA,
  // which a smaller launch leaves unpaired (1.03 ms unsplit, 1.24 in two).
  static_assert(kPieces >= 1 && kPieces <= 4, "events per net");
  const int halves = count >= kSplitMin && n->game == GZ_GAME_CHESS ? kPieces : 1;
  int first[5];
  for (int h = 0; h < halves; ++h) first[h] = count * h / halves / 6 * 6;
  first[halves] = count;
  auto issue = [&](const int8_t* src_b, const int8_t* src_s, int h) -> gz_status {
    const size_t lo = first[h], m = first[h + 1] - first[h];
    GZ_CUDA(cudaMemcpyAsync(d_boards + lo * s.board_bytes, src_b + lo * s.board_bytes, m * s.board_bytes,
                            cudaMemcpyHostToDevice, n->copy_stream));
    GZ_CUDA(cudaMemcpyAsync(d_side + lo, src_s + lo, m, cudaMemcpyHostToDevice, n->copy_stream));
    GZ_CUDA(cudaEventRecord(n->ev_in[h], n->copy_stream));
    GZ_CUDA(cudaStreamWaitEvent(n->stream, n->ev_in[h], 0));
    gz_status st = run_forward(n, d_boards + lo * s.board_bytes, d_side + lo, (int)m, d_pi + lo * s.actions, d_v + lo,
                               n->stream);
    if (st != GZ_OK) {
      cudaStreamSynchronize(n->copy_stream);  // no copy left reading the caller's or the staging buffers
      return st;
    }
    GZ_CUDA(cudaEventRecord(n->ev_fwd[h], n->stream));
    return GZ_OK;
  };
  auto collect = [&](float* dst_pi, float* dst_v, int h) -> gz_status {
    const size_t lo = first[h], m = first[h + 1] - first[h];
    GZ_CUDA(cudaStreamWaitEvent(n->copy_stream, n->ev_fwd[h], 0));
    GZ_CUDA(cudaMemcpyAsync(dst_pi + lo * s.actions, d_pi + lo * s.actions, m * s.actions * sizeof(float),
                            cudaMemcpyDeviceToHost, n->copy_stream));
    GZ_CUDA(cudaMemcpyAsync(dst_v + lo, d_v + lo, m * sizeof(float), cudaMemcpyDeviceToHost, n->copy_stream));
    if (h == halves - 1) GZ_CUDA(cudaMemcpyAsync(h_err, n->d_err, sizeof(int), cudaMemcpyDeviceToHost, n->copy_stream));
    GZ_CUDA(cudaEventRecord(n->ev_out[h], n->copy_stream));
    return GZ_OK;
  };

  if (halves == 1) {
    // Connect4 (small inputs and outputs) from mapped page-locked buffers:
    // the forward kernel reads the boards and writes the results through the
    // mapped addresses itself (one launch instead of five copies and a
    // launch; the same bytes cross the bus)
    void* mb = mapped_address(boards);
    void* ms = mb ? mapped_address(side) : nullptr;
    void* mp = ms ? mapped_address(pi) : nullptr;
    void* mv = mp ? mapped_address(v) : nullptr;
    if (mv) {
      if (gz_status st = run_forward(n, (const int8_t*)mb, (const int8_t*)ms, count, (float*)mp, (float*)mv, n->stream);
          st != GZ_OK) {
        cudaStreamSynchronize(n->stream);
        return st;
      }
      GZ_CUDA(cudaMemcpyAsync(h_err, n->d_err, sizeof(int), cudaMemcpyDeviceToHost, n->stream));
      GZ_CUDA(cudaStreamSynchronize(n->stream));
      return forward_error(n, *h_err);
    }
  }
  if (page_locked(boards) && page_locked(side) && page_locked(pi) && page_locked(v)) {
    // caller buffers are page-locked: the copy engines read and write them directly
    for (int h = 0; h < halves; ++h)
      if (gz_status st = issue(boards, side, h); st != GZ_OK) return st;
    for (int h = 0; h < halves; ++h)
      if (gz_status st = collect(pi, v, h); st != GZ_OK) return st;
    GZ_CUDA(cudaStreamSynchronize(n->copy_stream));
    return forward_error(n, *h_err);
  }

  // Pageable caller buffers go through the page-locked staging buffers; the
  // host copies of one half overlap the other half's transfers and forward
  // pass.
  int8_t* h_boards = n->h_in;
  int8_t* h_side = n->h_in + bb;
  float* h_pi = n->h_out;
  float* h_v = n->h_out + (size_t)count * s.actions;
  for (int h = 0; h < halves; ++h) {
    const size_t lo = first[h], m = first[h + 1] - first[h];
    memcpy(h_boards + lo * s.board_bytes, boards + lo * s.board_bytes, m * s.board_bytes);
    memcpy(h_side + lo, side + lo, m);
    if (gz_status st = issue(h_boards, h_side, h); st != GZ_OK) return st;
  }
  for (int h = 0; h < halves; ++h)
    if (gz_status st = collect(h_pi, h_v, h); st != GZ_OK) return st;
  for (int h = 0; h < halves; ++h) {
    const size_t lo = first[h], m = first[h + 1] - first[h];
    GZ_CUDA(cudaEventSynchronize(n->ev_out[h]));
    memcpy(pi + lo * s.actions, h_pi + lo * s.actions, m * s.actions * sizeof(float));
    memcpy(v + lo, h_v + lo, m * sizeof(float));
  }
  return forward_error(n, *h_err);
}

gz_status gz_net_predict(gz_net* n, const float* h_board, float* h_pi, float* h_v) {
  if (!n || !h_board || !h_pi || !h_v) return fail(GZ_ERR_INVALID_ARG, "null argument");
  if (n->game == kChess) return fail(GZ_ERR_UNSUPPORTED, "single-position chess boards need the full position record");
  GameShape s = game_shape(n->game);
  // Canonical board: own stones +1.  The side to move is the first player
  // iff both players have placed the same number of stones.
  int own = 0, opp = 0;
  for (int i = 0; i < s.nodes; ++i) {
    float x = h_board[i];
    if (x != 0.f && x != 1.f && x != -1.f) return fail(GZ_ERR_INVALID_ARG, "board cell %d = %g not in {-1,0,1}", i, x);
    own += x == 1.f;
    opp += x == -1.f;
  }
  int8_t side = own == opp ? 1 : -1;
  int8_t b[64];
  for (int i = 0; i < s.nodes; ++i) b[i] = (int8_t)((int)h_board[i] * side);
  return gz_net_predict_host(n, b, &side, 1, h_pi, h_v);
}

gz_status gz_nccl_unique_id(uint8_t out[128]) {
  Nccl* c = nccl();
  if (!c) return fail(GZ_ERR_NCCL, "libnccl.so.2 not loadable");
  if (!out) return fail(GZ_ERR_INVALID_ARG, "null id");
  ncclUniqueId id;
  ncclResult_t r = c->getUniqueId(&id);
  if (r != ncclSuccess) return fail(GZ_ERR_NCCL, "ncclGetUniqueId: %d", (int)r);
  static_assert(sizeof(id) == 128, "ncclUniqueId size");
  memcpy(out, &id, 128);
  return GZ_OK;
}

gz_status gz_nccl_comm_init(const uint8_t id_bytes[128], int world, int rank, int device, void** comm) {
  Nccl* c = nccl();
  if (!c) return fail(GZ_ERR_NCCL, "libnccl.so.2 not loadable");
  if (!id_bytes || !comm || world <= 0 || rank < 0 || rank >= world) return fail(GZ_ERR_INVALID_ARG, "bad arguments");
  GZ_DEVICE(device);
  ncclUniqueId id;
  memcpy(&id, id_bytes, 128);
  ncclComm_t cm = nullptr;
  ncclResult_t r = c->commInitRank(&cm, world, id, rank);
  if (r != ncclSuccess) return fail(GZ_ERR_NCCL, "ncclCommInitRank: %s", c->errorString ? c->errorString(r) : "?");
  *comm = cm;
  return GZ_OK;
}

gz_status gz_nccl_comm_destroy(void* comm) {
  Nccl* c = nccl();
  if (!c) return fail(GZ_ERR_NCCL, "libnccl.so.2 not loadable");
  if (comm) c->commDestroy((ncclComm_t)comm);
  return GZ_OK;
}

gz_status gz_net_broadcast(gz_net* n, void* comm, int root, void* stream) {
  if (!n || !comm) return fail(GZ_ERR_INVALID_ARG, "null argument");
  Nccl* c = nccl();
  if (!c) return fail(GZ_ERR_NCCL, "libnccl.so.2 not loadable");
  GZ_DEVICE(n->device);
  cudaStream_t s = (cudaStream_t)stream;
  ncclResult_t r = c->broadcast(n->d_weights, n->d_weights, n->weight_count, ncclFloat32, root, (ncclComm_t)comm, s);
  if (r != ncclSuccess) return fail(GZ_ERR_NCCL, "ncclBroadcast: %s", c->errorString ? c->errorString(r) : "?");
  return prepare_weights(n, s);
}

}  // extern "C"

int gz::net_game(const gz_net* n) { return n ? n->game : -1; }

gz_status gz::nccl_broadcast_floats(void* comm, float* d_buf, size_t count, int root, void* stream) {
  Nccl* c = nccl();
  if (!c) return fail(GZ_ERR_NCCL, "libnccl.so.2 not loadable");
  if (!comm) return fail(GZ_ERR_INVALID_ARG, "null communicator");
  const ncclResult_t r = c->broadcast(d_buf, d_buf, count, ncclFloat32, root, (ncclComm_t)comm, (cudaStream_t)stream);
  if (r != ncclSuccess) return fail(GZ_ERR_NCCL, "ncclBroadcast: %s", c->errorString ? c->errorString(r) : "?");
  return GZ_OK;
}

extern "C" {

// ---------------------------------------------------------------- training --
namespace {

gz_status ensure_train(gz_net* n, int batch) {
  if (batch <= 0) return fail(GZ_ERR_INVALID_ARG, "batch of %d positions", batch);
  if (!n->tr) n->tr = new gz::train::State();
  const cudaError_t e = n->kind == GZ_NET_RESNET ? gz::train::res_ensure_state(*n->tr, batch)
                                                 : gz::train::ensure_state(*n->tr, n->game, batch);
  if (e != cudaSuccess)
    return fail(GZ_ERR_CUDA, "training buffers for %d positions: %s", batch, cudaGetErrorString(e));
  return GZ_OK;
}

bool valid_train_config(const gz_train_config* c) {
  return c && c->batch_size > 0 && c->epochs >= 0 && c->learning_rate >= 0.f && c->weight_decay >= 0.f &&
         c->beta1 >= 0.f && c->beta1 < 1.f && c->beta2 >= 0.f && c->beta2 < 1.f && c->eps > 0.f;
}

// Forward + backward of one batch on `s`; with a communicator the gradient
// buckets are summed over the ranks on the training state's side stream as
// the backward pass completes them; with `update` an Adam step (gradients
// averaged over the ranks) and a repack of the tensor-core weights follow.
gz_status train_batch(gz_net* n, const int8_t* boards, const int8_t* side, const float* pi, const float* v, int cnt,
                      const gz_train_config* cfg, void* comm, int world, bool update, float* h_loss,
                      cudaStream_t s) {
  gz::train::State& st = *n->tr;
  Nccl* c = nullptr;
  if (comm && world > 1) {
    c = nccl();
    if (!c || !c->allReduce) return fail(GZ_ERR_NCCL, "libnccl.so.2 not loadable");
  }
  ncclResult_t nr = ncclSuccess;
  auto bucket_done = [&](int k) -> cudaError_t {
    if (!c) return cudaSuccess;
    cudaError_t e = cudaEventRecord(st.ev_bucket[k], s);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(st.comm_stream, st.ev_bucket[k], 0);
    if (e != cudaSuccess) return e;
    size_t off = 0, count = 0;
    if (n->kind == GZ_NET_RESNET)
      gz::train::res_bucket_range(k, &off, &count);
    else
      gz::train::bucket_range(n->game, k, &off, &count);
    if (nr == ncclSuccess)
      nr = c->allReduce(st.grad + off, st.grad + off, count, ncclFloat32, ncclSum, (ncclComm_t)comm, st.comm_stream);
    return cudaSuccess;
  };
  const cudaError_t e =
      n->kind == GZ_NET_RESNET
          ? gz::train::res_loss_and_grad(st, n->d_weights, boards, side, pi, v, cnt, s, bucket_done)
          : gz::train::loss_and_grad(st, n->d_weights, boards, side, pi, v, cnt, s, bucket_done);
  if (e != cudaSuccess) return fail(GZ_ERR_CUDA, "training step: %s", cudaGetErrorString(e));
  if (nr != ncclSuccess) return fail(GZ_ERR_NCCL, "ncclAllReduce: %s", c->errorString ? c->errorString(nr) : "?");
  if (c) {
    GZ_CUDA(cudaEventRecord(st.ev_comm, st.comm_stream));
    GZ_CUDA(cudaStreamWaitEvent(s, st.ev_comm, 0));
  }
  if (update) {
    const gz::train::AdamParams p{cfg->learning_rate, cfg->beta1, cfg->beta2, cfg->eps, cfg->weight_decay,
                                  c ? 1.f / (float)world : 1.f};
    GZ_CUDA(n->kind == GZ_NET_RESNET ? gz::train::res_adam_step(st, n->d_weights, p, s)
                                     : gz::train::adam_step(st, n->d_weights, p, s));
    const gz_status ps = prepare_weights(n, s);
    if (ps != GZ_OK) return ps;
  }
  if (h_loss) GZ_CUDA(cudaMemcpyAsync(h_loss, st.loss, 2 * sizeof(float), cudaMemcpyDeviceToHost, s));
  GZ_CUDA(cudaStreamSynchronize(s));
  return GZ_OK;
}

// Example order of pass `epoch`: a Fisher-Yates shuffle of 0 .. n-1 from a
// splitmix64 stream of (seed, epoch).
void epoch_order(int64_t n, uint64_t seed, int epoch, std::vector<int64_t>& order) {
  order.resize((size_t)n);
  for (int64_t i = 0; i < n; ++i) order[(size_t)i] = i;
  SplitMix r(mix_seed(seed, 0x7A1ull + (uint64_t)epoch));
  for (int64_t i = n - 1; i > 0; --i) {
    const int64_t j = (int64_t)(r.next() % (uint64_t)(i + 1));
    std::swap(order[(size_t)i], order[(size_t)j]);
  }
}

}  // namespace

void gz_train_config_default(gz_train_config* c) {
  if (!c) return;
  c->learning_rate = 1e-3f;
  c->weight_decay = 1e-4f;
  c->beta1 = 0.9f;
  c->beta2 = 0.999f;
  c->eps = 1e-8f;
  c->batch_size = 64;
  c->epochs = 10;
  c->seed = 0x6A5Aull;
}

gz_status gz_net_loss_grad(gz_net* n, const int8_t* d_boards, const int8_t* d_side, const float* d_pi,
                           const float* d_v, int cnt, float* d_grad, float h_loss[2], void* stream) {
  if (!n || (cnt > 0 && (!d_boards || !d_side || !d_pi || !d_v))) return fail(GZ_ERR_INVALID_ARG, "null argument");
  if (cnt <= 0) return fail(GZ_ERR_INVALID_ARG, "batch of %d positions", cnt);
  GZ_DEVICE(n->device);
  gz_status st = ensure_train(n, cnt);
  if (st != GZ_OK) return st;
  cudaStream_t s = (cudaStream_t)stream;
  st = train_batch(n, d_boards, d_side, d_pi, d_v, cnt, nullptr, nullptr, 1, false, h_loss, s);
  if (st != GZ_OK) return st;
  if (d_grad) {
    GZ_CUDA(cudaMemcpyAsync(d_grad, n->tr->grad, n->weight_count * sizeof(float), cudaMemcpyDeviceToDevice, s));
    GZ_CUDA(cudaStreamSynchronize(s));
  }
  return GZ_OK;
}

gz_status gz_net_train_step(gz_net* n, const int8_t* d_boards, const int8_t* d_side, const float* d_pi,
                            const float* d_v, int cnt, const gz_train_config* cfg, void* comm, int world,
                            float h_loss[2], void* stream) {
  if (!n || (cnt > 0 && (!d_boards || !d_side || !d_pi || !d_v))) return fail(GZ_ERR_INVALID_ARG, "null argument");
  if (!valid_train_config(cfg)) return fail(GZ_ERR_INVALID_ARG, "bad training configuration");
  if (cnt <= 0 || world < 1) return fail(GZ_ERR_INVALID_ARG, "batch of %d positions, world %d", cnt, world);
  GZ_DEVICE(n->device);
  const gz_status st = ensure_train(n, cnt);
  if (st != GZ_OK) return st;
  return train_batch(n, d_boards, d_side, d_pi, d_v, cnt, cfg, comm, world, true, h_loss, (cudaStream_t)stream);
}

gz_status gz_train_batch_indices(int64_t n, const gz_train_config* cfg, int epoch, int64_t step, int rank, int world,
                                 int64_t* out) {
  if (!valid_train_config(cfg) || !out || world < 1 || rank < 0 || rank >= world || epoch < 0 || step < 0)
    return fail(GZ_ERR_INVALID_ARG, "bad arguments");
  const int64_t B = cfg->batch_size, block = B * world;
  if (n < 0 || (step + 1) * block > n)
    return fail(GZ_ERR_INVALID_ARG, "step %lld of a pass over %lld examples (%lld per step)", (long long)step,
                (long long)n, (long long)block);
  std::vector<int64_t> order;
  epoch_order(n, cfg->seed, epoch, order);
  for (int64_t k = 0; k < B; ++k) out[k] = order[(size_t)(step * block + rank * B + k)];
  return GZ_OK;
}

gz_status gz_train_bucket_range(int game, int k, size_t* offset, size_t* count) {
  if (!valid_game(game) || !offset || !count || k < 0 || k >= gz::train::bucket_count(game))
    return fail(GZ_ERR_INVALID_ARG, "bad arguments");
  gz::train::bucket_range(game, k, offset, count);
  return GZ_OK;
}

gz_status gz_net_train(gz_net* n, const gz_train_example* ex, int64_t count, const gz_train_config* cfg, void* comm,
                       int rank, int world, gz_train_stats* stats) {
  if (!n || (count > 0 && !ex)) return fail(GZ_ERR_INVALID_ARG, "null argument");
  if (!valid_train_config(cfg)) return fail(GZ_ERR_INVALID_ARG, "bad training configuration");
  if (world < 1 || rank < 0 || rank >= world) return fail(GZ_ERR_INVALID_ARG, "rank %d of %d", rank, world);
  if (n->game != kTicTacToe && n->game != kConnect4)
    return fail(GZ_ERR_UNSUPPORTED, "training examples hold TicTacToe or Connect4 boards");
  GZ_DEVICE(n->device);
  const GameShape sh = game_shape(n->game);
  const int B = cfg->batch_size, A = sh.actions, N = sh.nodes;
  // canonical boards (own stones +1) -> board and side to move, as gz_net_predict
  std::vector<int8_t> boards((size_t)count * N), side((size_t)count);
  for (int64_t i = 0; i < count; ++i) {
    int own = 0, opp = 0;
    for (int k = 0; k < N; ++k) {
      const int x = ex[i].board[k];
      if (x < -1 || x > 1) return fail(GZ_ERR_INVALID_ARG, "example %lld: cell %d = %d", (long long)i, k, x);
      own += x == 1;
      opp += x == -1;
    }
    const int sd = own == opp ? 1 : -1;
    side[(size_t)i] = (int8_t)sd;
    for (int k = 0; k < N; ++k) boards[(size_t)i * N + k] = (int8_t)(ex[i].board[k] * sd);
  }
  const int64_t steps = count / ((int64_t)B * world);
  gz_status st = ensure_train(n, B);
  if (st != GZ_OK) return st;
  // per-step staging: host (page-locked) and device
  const size_t bytes = (size_t)B * (N + 1) + (size_t)B * (A + 1) * sizeof(float);
  uint8_t *h = nullptr, *d = nullptr;
  GZ_CUDA(cudaMallocHost(&h, bytes));
  if (cudaMalloc(&d, bytes) != cudaSuccess) {
    cudaFreeHost(h);
    return fail(GZ_ERR_CUDA, "cudaMalloc of %zu bytes of training staging", bytes);
  }
  int8_t* hb = (int8_t*)h;
  int8_t* hs = hb + (size_t)B * N;
  float* hp = (float*)(h + (size_t)B * (N + 1));
  float* hv = hp + (size_t)B * A;
  const size_t off_pi = (size_t)B * (N + 1);
  float ploss = 0.f, vloss = 0.f;
  std::vector<int64_t> order;
  for (int ep = 0; ep < cfg->epochs && st == GZ_OK; ++ep) {
    epoch_order(count, cfg->seed, ep, order);
    double sp = 0.0, sv = 0.0;
    for (int64_t k = 0; k < steps && st == GZ_OK; ++k) {
      for (int j = 0; j < B; ++j) {
        const int64_t i = order[(size_t)(k * B * world + (int64_t)rank * B + j)];
        memcpy(hb + (size_t)j * N, boards.data() + (size_t)i * N, (size_t)N);
        hs[j] = side[(size_t)i];
        memcpy(hp + (size_t)j * A, ex[i].pi, (size_t)A * sizeof(float));
        hv[j] = ex[i].v;
      }
      float loss[2] = {0.f, 0.f};
      if (cudaMemcpyAsync(d, h, bytes, cudaMemcpyHostToDevice, n->stream) != cudaSuccess) {
        st = fail(GZ_ERR_CUDA, "training batch upload");
        break;
      }
      st = train_batch(n, (const int8_t*)d, (const int8_t*)(d + (size_t)B * N), (const float*)(d + off_pi),
                       (const float*)(d + off_pi) + (size_t)B * A, B, cfg, comm, world, true, loss, n->stream);
      sp += loss[0];
      sv += loss[1];
    }
    if (steps > 0) {
      ploss = (float)(sp / (double)steps);
      vloss = (float)(sv / (double)steps);
    }
  }
  cudaFreeHost(h);
  cudaFree(d);
  if (stats) {
    stats->policy_loss = ploss;
    stats->value_loss = vloss;
    stats->steps = n->tr->step;
  }
  return st;
}

// ------------------------------------------------------ failure detection --
namespace {
// Waits on an mbarrier nothing arrives at; reports through *status:
// 1 = the bounded wait gave up (expected), 0 = it completed.
__global__ void wait_timeout_kernel(int* status, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    gz::sm100::mbar_init(&bar, 1);
    abort_flag = 0;
    gz::sm100::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool ok = gz::sm100::mbar_wait(&bar, 0, (volatile int*)&abort_flag, limit_ns);
    *status = ok ? 0 : 1;
  }
}
}  // namespace

gz_status gz_selftest_wait_timeout(int device, int limit_us) {
  if (limit_us <= 0 || limit_us > 10000000) return fail(GZ_ERR_INVALID_ARG, "limit_us out of range");
  GZ_DEVICE(device);
  int* d = nullptr;
  GZ_CUDA(cudaMalloc(&d, sizeof(int)));
  GZ_CUDA(cudaMemset(d, 0xFF, sizeof(int)));
  wait_timeout_kernel<<<1, 32>>>(d, (unsigned long long)limit_us * 1000ull);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  int st = -1;
  if (e == cudaSuccess) e = cudaMemcpy(&st, d, sizeof(int), cudaMemcpyDeviceToHost);
  cudaFree(d);
  if (e != cudaSuccess) return fail(GZ_ERR_CUDA, "selftest: %s", cudaGetErrorString(e));
  if (st == 1) return fail(GZ_ERR_TIMEOUT, "bounded wait gave up after %d us (expected)", limit_us);
  if (st == 0) return GZ_OK;
  return fail(GZ_ERR_CUDA, "selftest kernel did not report");
}

// ---------------------------------------------------------------- search --
gz_status gz_mcts_create(const gz_mcts_config* cfg, int device, gz_mcts** out) {
  if (!cfg || !out) return fail(GZ_ERR_INVALID_ARG, "null argument");
  *out = nullptr;
  if (!valid_game(cfg->game)) return fail(GZ_ERR_INVALID_ARG, "bad game %d", cfg->game);
  if (cfg->trees <= 0 || cfg->leaves_per_tree <= 0 || cfg->node_capacity < 2 || cfg->virtual_loss < 0)
    return fail(GZ_ERR_INVALID_ARG, "bad search sizes");
  if (!(cfg->c_puct >= 0.f) || !(cfg->dirichlet_eps >= 0.f && cfg->dirichlet_eps <= 1.f) ||
      (cfg->dirichlet_eps > 0.f && !(cfg->dirichlet_alpha > 0.f)))
    return fail(GZ_ERR_INVALID_ARG, "bad search constants");
  int ndev = 0;
  GZ_CUDA(cudaGetDeviceCount(&ndev));
  if (device < 0 || device >= ndev) return fail(GZ_ERR_INVALID_ARG, "device %d of %d", device, ndev);
  GZ_DEVICE(device);
  gz_mcts* m = new gz_mcts();
  m->device = device;
  MctsDev& d = m->d;
  GameShape s = game_shape(cfg->game);
  d.game = cfg->game;
  d.trees = cfg->trees;
  d.leaves = cfg->leaves_per_tree;
  d.vl_k = cfg->virtual_loss;
  d.node_cap = cfg->node_capacity;
  // every node's edges fit: TicTacToe and Connect4 reserve an edge per
  // action; a chess node averages about 35 legal moves (at most 218), so the
  // pool reserves 64 per node and a search that outgrows it reports
  // kMctsEdgeCap through gz_mcts_check
  d.edge_cap = cfg->node_capacity * (cfg->game == kChess ? 64 : s.actions);
  d.N = s.nodes;
  d.board_bytes = s.board_bytes;
  d.A = s.actions;
  d.c_puct = cfg->c_puct;
  d.dir_alpha = cfg->dirichlet_alpha;
  d.dir_eps = cfg->dirichlet_eps;
  d.seed = cfg->seed;
  const size_t T = (size_t)d.trees, EC = T * d.edge_cap, L = T * d.leaves;
  gz_status st = GZ_OK;
  auto alloc = [&](auto** p, size_t bytes) {
    if (st != GZ_OK) return;
    cudaError_t e = cudaMalloc((void**)p, bytes ? bytes : 1);
    if (e != cudaSuccess) st = fail(GZ_ERR_CUDA, "cudaMalloc %zu bytes: %s", bytes, cudaGetErrorString(e));
    else m->allocs.push_back((void*)*p);
  };
  alloc(&d.tree, T * sizeof(MctsTree));
  alloc(&d.edges, EC * sizeof(MctsEdge));
  alloc(&d.path_edges, L * kMctsMaxDepth * 4); alloc(&d.path_len, L * 4); alloc(&d.leaf_legal, L * 4);
  alloc(&d.leaf_board, L * d.board_bytes); alloc(&d.leaf_side, L); alloc(&d.leaf_terminal, L);
  if (d.game == kChess) {
    alloc(&d.ctree, T * sizeof(ChessTree));
    alloc(&d.leaf_actions, L * kChessMaxLegal * sizeof(int16_t));
    alloc(&d.leaf_count, L * 4);
  }
  alloc(&d.err, 4);
  alloc(&m->d_pi, L * d.A * 4); alloc(&m->d_v, L * 4);
  alloc(&m->d_tmp, T * 4 * 2);
  if (st == GZ_OK) {
    // empty roots (no position loaded: an all-zero board, first player to move)
    std::vector<MctsTree> h(T);
    for (MctsTree& tr : h) {
      memset(&tr, 0, sizeof tr);
      tr.fe = -1;
      tr.meta = (uint32_t)kNodeCreated << 16;
      tr.node_count = 1;
      tr.side = 1;
    }
    cudaError_t e = cudaMemset(d.err, 0, 4);
    if (e == cudaSuccess) e = cudaMemcpy(d.tree, h.data(), T * sizeof(MctsTree), cudaMemcpyHostToDevice);
    if (e == cudaSuccess && d.game == kChess) {  // chess roots start at the initial position
      std::vector<ChessTree> hc(T);
      chess::Pos p0;
      chess::start_pos(p0);
      for (ChessTree& tr : hc) {
        memset(&tr, 0, sizeof tr);
        chess::to_record(p0, tr.rec);
        tr.side = 1;
        tr.fe = -1;
        tr.meta = (uint32_t)kNodeCreated << 16;
        tr.node_count = 1;
      }
      e = cudaMemcpy(d.ctree, hc.data(), T * sizeof(ChessTree), cudaMemcpyHostToDevice);
      if (e == cudaSuccess) e = cudaMemset(d.leaf_count, 0, L * 4);
    }
    if (e == cudaSuccess) e = cudaMemset(d.path_len, 0, L * 4);
    if (e == cudaSuccess) e = cudaMemset(d.path_edges, 0, L * kMctsMaxDepth * 4);
    if (e == cudaSuccess) e = cudaMemset(d.leaf_legal, 0, L * 4);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) st = fail(GZ_ERR_CUDA, "init: %s", cudaGetErrorString(e));
  }
  if (st != GZ_OK) {
    gz_mcts_destroy(m);
    return st;
  }
  *out = m;
  return GZ_OK;
}

gz_status gz_mcts_destroy(gz_mcts* m) {
  if (!m) return GZ_OK;
  DeviceGuard g(m->device);
  cudaDeviceSynchronize();
  for (void* p : m->allocs) cudaFree(p);
  delete m;
  return GZ_OK;
}

gz_status gz_mcts_reset_roots(gz_mcts* m, const int8_t* boards, const int8_t* side, void* stream) {
  if (!m || !boards || !side) return fail(GZ_ERR_INVALID_ARG, "null argument");
  GZ_DEVICE(m->device);
  GZ_CUDA(mcts_launch_reset(m->d, boards, side, (cudaStream_t)stream));
  return GZ_OK;
}

gz_status gz_mcts_select(gz_mcts* m, void* stream) {
  if (!m) return fail(GZ_ERR_INVALID_ARG, "null argument");
  GZ_DEVICE(m->device);
  GZ_CUDA(mcts_launch_select(m->d, (cudaStream_t)stream));
  return GZ_OK;
}

gz_status gz_mcts_leaf_buffers(gz_mcts* m, int8_t** boards, int8_t** side, int8_t** terminal) {
  if (!m) return fail(GZ_ERR_INVALID_ARG, "null argument");
  if (boards) *boards = m->d.leaf_board;
  if (side) *side = m->d.leaf_side;
  if (terminal) *terminal = m->d.leaf_terminal;
  return GZ_OK;
}

gz_status gz_mcts_copy_leaves(gz_mcts* m, int8_t* boards, int8_t* side, int8_t* terminal, void* stream) {
  if (!m) return fail(GZ_ERR_INVALID_ARG, "null argument");
  GZ_DEVICE(m->device);
  cudaStream_t s = (cudaStream_t)stream;
  size_t L = (size_t)m->d.trees * m->d.leaves;
  if (boards) GZ_CUDA(cudaMemcpyAsync(boards, m->d.leaf_board, L * m->d.board_bytes, cudaMemcpyDeviceToHost, s));
  if (side) GZ_CUDA(cudaMemcpyAsync(side, m->d.leaf_side, L, cudaMemcpyDeviceToHost, s));
  if (terminal) GZ_CUDA(cudaMemcpyAsync(terminal, m->d.leaf_terminal, L, cudaMemcpyDeviceToHost, s));
  GZ_CUDA(cudaStreamSynchronize(s));
  return GZ_OK;
}

gz_status gz_mcts_backup(gz_mcts* m, const float* pi, const float* v, void* stream) {
  if (!m || !pi || !v) return fail(GZ_ERR_INVALID_ARG, "null argument");
  GZ_DEVICE(m->device);
  GZ_CUDA(mcts_launch_backup(m->d, pi, v, (cudaStream_t)stream));
  return GZ_OK;
}

gz_status gz_mcts_step(gz_mcts* m, gz_net* net, void* stream) {
  if (!m || !net) return fail(GZ_ERR_INVALID_ARG, "null argument");
  if (net->game != m->d.game) return fail(GZ_ERR_INVALID_ARG, "net and search play different games");
  if (net->device != m->device) return fail(GZ_ERR_INVALID_ARG, "net and search live on different devices");
  GZ_DEVICE(m->device);
  cudaStream_t s = (cudaStream_t)stream;
  GZ_CUDA(mcts_launch_select(m->d, s));
  gz_status st = run_forward(net, m->d.leaf_board, m->d.leaf_side, m->d.trees * m->d.leaves, m->d_pi, m->d_v, s);
  if (st != GZ_OK) return st;
  GZ_CUDA(mcts_launch_backup(m->d, m->d_pi, m->d_v, s));
  return GZ_OK;
}

gz_status gz_mcts_run(gz_mcts* m, gz_net* net, int sims, void* stream) {
  if (!m || !net || sims < 0) return fail(GZ_ERR_INVALID_ARG, "bad arguments");
  if (net->game != m->d.game) return fail(GZ_ERR_INVALID_ARG, "net and search play different games");
  if (net->device != m->device) return fail(GZ_ERR_INVALID_ARG, "net and search live on different devices");
  const int waves = (sims + m->d.leaves - 1) / m->d.leaves;
  if (waves == 0) return GZ_OK;
  GZ_DEVICE(m->device);
  cudaStream_t s = (cudaStream_t)stream;
  // the gz_mcts_step sequence, with each backup and the next selections in one launch
  GZ_CUDA(mcts_launch_select(m->d, s));
  for (int w = 0; w < waves; ++w) {
    gz_status st = run_forward(net, m->d.leaf_board, m->d.leaf_side, m->d.trees * m->d.leaves, m->d_pi, m->d_v, s);
    if (st != GZ_OK) return st;
    if (w + 1 < waves) GZ_CUDA(mcts_launch_backup_select(m->d, m->d_pi, m->d_v, s));
    else GZ_CUDA(mcts_launch_backup(m->d, m->d_pi, m->d_v, s));
  }
  return GZ_OK;
}

gz_status gz_mcts_check(gz_mcts* m) {
  if (!m) return fail(GZ_ERR_INVALID_ARG, "null argument");
  GZ_DEVICE(m->device);
  int err = 0;
  GZ_CUDA(cudaMemcpy(&err, m->d.err, 4, cudaMemcpyDeviceToHost));
  if (err == kMctsNodeCap) return fail(GZ_ERR_CAPACITY, "search node pool exhausted (node_capacity %d)", m->d.node_cap);
  if (err == kMctsEdgeCap) return fail(GZ_ERR_CAPACITY, "search edge pool exhausted");
  if (err == kMctsDepth) return fail(GZ_ERR_CAPACITY, "search path deeper than %d", kMctsMaxDepth);
  return GZ_OK;
}

gz_status gz_mcts_root_stats(gz_mcts* m, int32_t* visits, float* wsum, void* stream) {
  if (!m || !visits) return fail(GZ_ERR_INVALID_ARG, "null argument");
  GZ_DEVICE(m->device);
  cudaStream_t s = (cudaStream_t)stream;
  size_t cnt = (size_t)m->d.trees * m->d.A;
  int32_t* dv = nullptr;
  float* dw = nullptr;
  GZ_CUDA(cudaMallocAsync((void**)&dv, cnt * 4, s));
  GZ_CUDA(cudaMallocAsync((void**)&dw, cnt * 4, s));
  GZ_CUDA(mcts_launch_root_visits(m->d, dv, dw, s));
  GZ_CUDA(cudaMemcpyAsync(visits, dv, cnt * 4, cudaMemcpyDeviceToHost, s));
  if (wsum) GZ_CUDA(cudaMemcpyAsync(wsum, dw, cnt * 4, cudaMemcpyDeviceToHost, s));
  GZ_CUDA(cudaFreeAsync(dv, s));
  GZ_CUDA(cudaFreeAsync(dw, s));
  GZ_CUDA(cudaStreamSynchronize(s));
  return gz_mcts_check(m);
}

gz_status gz_mcts_tree_sizes(gz_mcts* m, int32_t* nodes, int32_t* edges, void* stream) {
  if (!m || !nodes || !edges) return fail(GZ_ERR_INVALID_ARG, "null argument");
  GZ_DEVICE(m->device);
  cudaStream_t s = (cudaStream_t)stream;
  GZ_CUDA(mcts_launch_tree_sizes(m->d, m->d_tmp, m->d_tmp + m->d.trees, s));
  GZ_CUDA(cudaMemcpyAsync(nodes, m->d_tmp, (size_t)m->d.trees * 4, cudaMemcpyDeviceToHost, s));
  GZ_CUDA(cudaMemcpyAsync(edges, m->d_tmp + m->d.trees, (size_t)m->d.trees * 4, cudaMemcpyDeviceToHost, s));
  GZ_CUDA(cudaStreamSynchronize(s));
  return GZ_OK;
}

gz_status gz_mcts_choose(gz_mcts* m, int temp_moves, int32_t* actions, void* stream) {
  if (!m || !actions) return fail(GZ_ERR_INVALID_ARG, "null argument");
  GZ_DEVICE(m->device);
  GZ_CUDA(mcts_launch_choose(m->d, temp_moves, actions, (cudaStream_t)stream));
  return GZ_OK;
}

gz_status gz_mcts_play(gz_mcts* m, const int32_t* actions, int reserve, int8_t* done, void* stream) {
  if (!m || !actions || reserve < 0) return fail(GZ_ERR_INVALID_ARG, "bad arguments");
  GZ_DEVICE(m->device);
  GZ_CUDA(mcts_launch_play(m->d, actions, reserve, done, (cudaStream_t)stream));
  return GZ_OK;
}

// ---- self-play ----

static_assert(sizeof(gz_train_example) == 516, "TrainingExample layout of self_play/self_play.cuh:56-60");

gz_status gz_selfplay_create(gz_mcts* m, int max_examples, gz_selfplay** out) {
  if (!m || !out || max_examples <= 0) return fail(GZ_ERR_INVALID_ARG, "bad arguments");
  *out = nullptr;
  if (m->d.game == kChess)
    return fail(GZ_ERR_UNSUPPORTED, "self-play records TicTacToe and Connect4 games (the 64-cell example format)");
  GZ_DEVICE(m->device);
  gz_selfplay* sp = new gz_selfplay();
  sp->m = m;
  sp->device = m->device;
  SelfPlayDev& s = sp->s;
  const MctsDev& d = m->d;
  s.max_moves = d.N;  // a game fills at most every cell, one example per move
  s.out_cap = max_examples;
  const size_t slots = (size_t)d.trees * s.max_moves;
  gz_status st = GZ_OK;
  auto alloc = [&](auto** p, size_t bytes) {
    if (st != GZ_OK) return;
    cudaError_t e = cudaMalloc((void**)p, bytes ? bytes : 1);
    if (e != cudaSuccess) st = fail(GZ_ERR_CUDA, "cudaMalloc %zu bytes: %s", bytes, cudaGetErrorString(e));
    else sp->allocs.push_back((void*)*p);
  };
  alloc(&s.log_board, slots * d.N);
  alloc(&s.log_pi, slots * d.A * 4);
  alloc(&s.log_v, slots * 4);
  alloc(&s.log_side, slots);
  alloc(&s.log_len, (size_t)d.trees * 4);
  alloc(&s.fin_len, (size_t)d.trees * 4);
  alloc(&s.out, (size_t)max_examples * sizeof(gz_train_example));
  alloc(&sp->d_counts, 3 * 4);
  alloc(&sp->d_actions, (size_t)d.trees * 4);
  if (st == GZ_OK) {
    s.out_count = sp->d_counts;
    s.games_done = sp->d_counts + 1;
    s.overflow = sp->d_counts + 2;
    cudaError_t e = cudaMemset(s.log_len, 0, (size_t)d.trees * 4);
    if (e == cudaSuccess) e = cudaMemset(sp->d_counts, 0, 3 * 4);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) st = fail(GZ_ERR_CUDA, "init: %s", cudaGetErrorString(e));
  }
  if (st != GZ_OK) {
    gz_selfplay_destroy(sp);
    return st;
  }
  *out = sp;
  return GZ_OK;
}

gz_status gz_selfplay_destroy(gz_selfplay* sp) {
  if (!sp) return GZ_OK;
  DeviceGuard g(sp->device);
  cudaDeviceSynchronize();
  for (void* p : sp->allocs) cudaFree(p);
  delete sp;
  return GZ_OK;
}

gz_status gz_selfplay_run(gz_selfplay* sp, gz_net* net, int n_games, int sims, int temp_moves, void* stream) {
  if (!sp || !net || n_games < 0 || sims <= 0) return fail(GZ_ERR_INVALID_ARG, "bad arguments");
  gz_mcts* m = sp->m;
  if (net->game != m->d.game) return fail(GZ_ERR_INVALID_ARG, "net and search play different games");
  if (net->device != m->device) return fail(GZ_ERR_INVALID_ARG, "net and search live on different devices");
  GZ_DEVICE(m->device);
  cudaStream_t s = (cudaStream_t)stream;
  int counts[3];
  GZ_CUDA(cudaMemcpyAsync(counts, sp->d_counts, sizeof counts, cudaMemcpyDeviceToHost, s));
  GZ_CUDA(cudaStreamSynchronize(s));
  const int target = counts[1] + n_games;
  // every tree ends a game at least every max_moves moves
  const long long max_moves = ((long long)n_games / m->d.trees + 2) * (sp->s.max_moves + 1);
  // keep a child's subtree while the next move's simulations fit in the pool
  const int reserve = sims + m->d.leaves;
  for (long long mv = 0; mv < max_moves && counts[1] < target; ++mv) {
    gz_status st = gz_mcts_run(m, net, sims, stream);
    if (st != GZ_OK) return st;
    GZ_CUDA(selfplay_launch_record(m->d, sp->s, temp_moves, s));
    GZ_CUDA(mcts_launch_choose(m->d, temp_moves, sp->d_actions, s));
    GZ_CUDA(selfplay_launch_finish(m->d, sp->s, sp->d_actions, s));
    GZ_CUDA(selfplay_launch_emit(m->d, sp->s, s));
    GZ_CUDA(mcts_launch_play(m->d, sp->d_actions, reserve, nullptr, s));
    GZ_CUDA(cudaMemcpyAsync(counts, sp->d_counts, sizeof counts, cudaMemcpyDeviceToHost, s));
    GZ_CUDA(cudaStreamSynchronize(s));
    if (counts[2]) break;
  }
  gz_status st = gz_mcts_check(m);
  if (st != GZ_OK) return st;
  if (counts[2] == 1) return fail(GZ_ERR_CAPACITY, "a game outgrew its example log");
  if (counts[2] == 2) return fail(GZ_ERR_CAPACITY, "example buffer full (%d examples): take them first", sp->s.out_cap);
  if (counts[1] < target) return fail(GZ_ERR_TIMEOUT, "games did not end within %lld moves", max_moves);
  return GZ_OK;
}

gz_status gz_selfplay_take(gz_selfplay* sp, gz_train_example* out, int64_t capacity, int64_t* n_examples,
                           int64_t* n_games) {
  if (!sp || (!out && capacity > 0) || capacity < 0) return fail(GZ_ERR_INVALID_ARG, "bad arguments");
  GZ_DEVICE(sp->device);
  int counts[3];
  GZ_CUDA(cudaMemcpy(counts, sp->d_counts, sizeof counts, cudaMemcpyDeviceToHost));
  if (n_examples) *n_examples = counts[0];
  if (n_games) *n_games = counts[1];
  if (counts[0] > capacity) return fail(GZ_ERR_CAPACITY, "%d examples buffered, room for %lld", counts[0], (long long)capacity);
  if (counts[0] > 0) GZ_CUDA(cudaMemcpy(out, sp->s.out, (size_t)counts[0] * sizeof(gz_train_example), cudaMemcpyDeviceToHost));
  GZ_CUDA(cudaMemset(sp->d_counts, 0, 3 * 4));
  return GZ_OK;
}

// ---- arena ----

gz_status gz_arena_play(gz_mcts* m, gz_net* net_a, gz_net* net_b, int n_games, int sims, int32_t* a_wins,
                        int32_t* b_wins, int32_t* draws, void* stream) {
  if (!m || !net_a || !net_b || n_games < 0 || sims <= 0 || !a_wins || !b_wins || !draws)
    return fail(GZ_ERR_INVALID_ARG, "bad arguments");
  if (m->d.game == kChess) return fail(GZ_ERR_UNSUPPORTED, "the arena plays TicTacToe and Connect4");
  if (net_a->game != m->d.game || net_b->game != m->d.game)
    return fail(GZ_ERR_INVALID_ARG, "nets and search play different games");
  if (net_a->device != m->device || net_b->device != m->device)
    return fail(GZ_ERR_INVALID_ARG, "nets and search live on different devices");
  GZ_DEVICE(m->device);
  cudaStream_t s = (cudaStream_t)stream;
  const MctsDev& d = m->d;
  const int T = d.trees, A = d.A, N = d.N;
  const size_t L = (size_t)T * d.leaves;
  // one scratch block: two networks' evaluations, game state, moves
  const size_t o_pib = L * A * 4, o_va = 2 * o_pib, o_vb = o_va + L * 4, o_act = o_vb + L * 4,
               o_cnt = o_act + (size_t)T * 4, o_brd = o_cnt + 16, o_side = o_brd + (size_t)T * N,
               o_amv = o_side + T, o_actv = o_amv + T, o_res = o_actv + T, bytes = o_res + T;
  uint8_t* buf = nullptr;
  GZ_CUDA(cudaMallocAsync((void**)&buf, bytes, s));
  float *pi_a = (float*)buf, *pi_b = (float*)(buf + o_pib), *v_a = (float*)(buf + o_va), *v_b = (float*)(buf + o_vb);
  int32_t* actions = (int32_t*)(buf + o_act);
  int* n_active = (int*)(buf + o_cnt);
  int8_t *boards = (int8_t*)(buf + o_brd), *side = (int8_t*)(buf + o_side), *a_moves = (int8_t*)(buf + o_amv),
         *active = (int8_t*)(buf + o_actv), *result = (int8_t*)(buf + o_res);
  std::vector<int8_t> h_side(T, 1), h_amv(T), h_act(T), h_res(T);
  const int waves = (sims + d.leaves - 1) / d.leaves;
  int wa = 0, wb = 0, dr = 0;
  gz_status st = GZ_OK;
  auto cuda = [&](cudaError_t e, const char* what) {
    if (st == GZ_OK && e != cudaSuccess) st = fail(GZ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return st == GZ_OK;
  };
  for (int g0 = 0; g0 < n_games && st == GZ_OK; g0 += T) {
    const int n = n_games - g0 < T ? n_games - g0 : T;
    for (int t = 0; t < T; ++t) {
      h_act[t] = t < n;
      h_amv[t] = g0 + t < n_games / 2;  // net A moves first in the first half (arena.cu:98-102)
    }
    cuda(cudaMemsetAsync(boards, 0, (size_t)T * N, s), "memset");
    cuda(cudaMemsetAsync(result, 0, T, s), "memset");
    cuda(cudaMemcpyAsync(side, h_side.data(), T, cudaMemcpyHostToDevice, s), "copy");
    cuda(cudaMemcpyAsync(a_moves, h_amv.data(), T, cudaMemcpyHostToDevice, s), "copy");
    cuda(cudaMemcpyAsync(active, h_act.data(), T, cudaMemcpyHostToDevice, s), "copy");
    int live = n;
    for (int mv = 0; live > 0 && mv <= N && st == GZ_OK; ++mv) {
      cuda(mcts_launch_reset(d, boards, side, s), "reset");
      if (waves > 0) cuda(mcts_launch_select(d, s), "select");
      for (int w = 0; w < waves && st == GZ_OK; ++w) {
        if (st == GZ_OK) st = run_forward(net_a, d.leaf_board, d.leaf_side, (int)L, pi_a, v_a, s);
        if (st == GZ_OK) st = run_forward(net_b, d.leaf_board, d.leaf_side, (int)L, pi_b, v_b, s);
        cuda(arena_launch_merge((int)L, d.leaves, A, a_moves, pi_a, v_a, pi_b, v_b, m->d_pi, m->d_v, s), "merge");
        if (w + 1 < waves) cuda(mcts_launch_backup_select(d, m->d_pi, m->d_v, s), "backup+select");
        else cuda(mcts_launch_backup(d, m->d_pi, m->d_v, s), "backup");
      }
      cuda(mcts_launch_choose(d, 0, actions, s), "choose");
      cuda(cudaMemsetAsync(n_active, 0, 4, s), "memset");
      cuda(arena_launch_play(d.game, T, N, boards, side, a_moves, active, actions, result, n_active, s), "play");
      cuda(cudaMemcpyAsync(&live, n_active, 4, cudaMemcpyDeviceToHost, s), "copy");
      cuda(cudaStreamSynchronize(s), "synchronize");
    }
    cuda(cudaMemcpyAsync(h_res.data(), result, T, cudaMemcpyDeviceToHost, s), "copy");
    cuda(cudaStreamSynchronize(s), "synchronize");
    for (int t = 0; t < n && st == GZ_OK; ++t) {
      wa += h_res[t] == 1;
      wb += h_res[t] == 2;
      dr += h_res[t] == 3;
    }
  }
  cudaFreeAsync(buf, s);
  cudaStreamSynchronize(s);
  if (st != GZ_OK) return st;
  if ((st = gz_mcts_check(m)) != GZ_OK) return st;
  if ((st = gz_net_check(net_a)) != GZ_OK) return st;
  if ((st = gz_net_check(net_b)) != GZ_OK) return st;
  if (wa + wb + dr != n_games) return fail(GZ_ERR_TIMEOUT, "%d of %d games did not end", n_games - wa - wb - dr, n_games);
  *a_wins = wa;
  *b_wins = wb;
  *draws = dr;
  return GZ_OK;
}

gz_status gz_train_examples_save(const char* path, int n_iters, const gz_train_example* const* iters,
                                 const int32_t* counts) {
  if (!path || n_iters < 0 || (n_iters > 0 && (!iters || !counts))) return fail(GZ_ERR_INVALID_ARG, "bad arguments");
  for (int i = 0; i < n_iters; ++i)
    if (counts[i] < 0 || (counts[i] > 0 && !iters[i])) return fail(GZ_ERR_INVALID_ARG, "bad iteration %d", i);
  FILE* f = fopen(path, "wb");
  if (!f) return fail(GZ_ERR_IO, "cannot open %s for writing", path);
  const int32_t h = n_iters;
  bool ok = fwrite(&h, 4, 1, f) == 1;
  for (int i = 0; i < n_iters && ok; ++i) {
    ok = fwrite(&counts[i], 4, 1, f) == 1;
    if (ok && counts[i] > 0) ok = fwrite(iters[i], sizeof(gz_train_example), (size_t)counts[i], f) == (size_t)counts[i];
  }
  ok = (fclose(f) == 0) && ok;
  return ok ? GZ_OK : fail(GZ_ERR_IO, "write to %s failed", path);
}

gz_status gz_train_examples_load(const char* path, gz_train_example* out, int64_t capacity, int32_t* counts,
                                 int max_iters, int* n_iters, int64_t* total) {
  if (!path || !n_iters || !total || capacity < 0 || (out && (!counts || max_iters < 0)))
    return fail(GZ_ERR_INVALID_ARG, "bad arguments");
  FILE* f = fopen(path, "rb");
  if (!f) return fail(GZ_ERR_IO, "cannot open %s", path);
  gz_status st = GZ_OK;
  int32_t h = 0;
  long long sum = 0;
  if (fread(&h, 4, 1, f) != 1 || h < 0) st = fail(GZ_ERR_IO, "%s: bad header", path);
  if (st == GZ_OK && out && h > max_iters) st = fail(GZ_ERR_CAPACITY, "%s holds %d iterations, room for %d", path, h, max_iters);
  for (int i = 0; i < h && st == GZ_OK; ++i) {
    int32_t c = 0;
    if (fread(&c, 4, 1, f) != 1 || c < 0) {
      st = fail(GZ_ERR_IO, "%s: bad count of iteration %d", path, i);
      break;
    }
    if (out) {
      if (sum + c > capacity) {
        st = fail(GZ_ERR_CAPACITY, "%s holds more than %lld examples", path, (long long)capacity);
        break;
      }
      if (c > 0 && fread(out + sum, sizeof(gz_train_example), (size_t)c, f) != (size_t)c) {
        st = fail(GZ_ERR_IO, "%s: short iteration %d", path, i);
        break;
      }
      counts[i] = c;
    } else if (c > 0 && fseek(f, (long)((size_t)c * sizeof(gz_train_example)), SEEK_CUR) != 0) {
      st = fail(GZ_ERR_IO, "%s: short iteration %d", path, i);
      break;
    }
    sum += c;
  }
  if (st == GZ_OK && !out) {  // a size query still checks that the records are all there
    const long pos = ftell(f);
    if (fseek(f, 0, SEEK_END) != 0 || ftell(f) < pos) st = fail(GZ_ERR_IO, "%s: short file", path);
  }
  fclose(f);
  if (st != GZ_OK) return st;
  *n_iters = h;
  *total = sum;
  return GZ_OK;
}

}  // extern "C"
