/*
 * graphzero_b200 — C ABI of the B200 leaf-evaluation and batched PUCT path.
 *
 * Drop-in boundary for GraphZero's INeuralNet (networks/neural_network.h:16-27)
 * and the leaf-evaluation call inside its search (self_play/self_play.cu:617-632).
 * Plain C types only: device pointers are raw addresses, streams are
 * cudaStream_t passed as void*, NCCL communicators as void*.
 *
 * Errors: every function returns gz_status and never exits the process (the
 * reference exits through CUDA_CHECK/NCCL_CHECK, networks/gat/gat.cu:16-25).
 * gz_last_error() returns a message for the calling thread's last failure.
 *
 * Threading: one gz_net / gz_mcts handle belongs to one device; calls on one
 * handle must be serialised by the caller.  Handles on different devices are
 * independent.
 *
 * Position encoding (int8): TicTacToe [9] and Connect4 [42] hold the cells
 * row-major with +1 for the first player, -1 for the second, 0 empty
 * (games/connect4/connect4.cu:22-34); chess [66] holds 64 squares with piece
 * codes +-1..6 = P N B R Q K (white positive, games/chess/chess.cuh:11-21),
 * a castling-rights byte (bit 0 WK, 1 WQ, 2 BK, 3 BQ) and the en-passant
 * square (-1 none).  side[i] is the player to move (+1 / -1).
 */
#ifndef GRAPHZERO_B200_H
#define GRAPHZERO_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  GZ_OK = 0,
  GZ_ERR_INVALID_ARG = 1,
  GZ_ERR_CUDA = 2,
  GZ_ERR_NCCL = 3,
  GZ_ERR_TIMEOUT = 4,
  GZ_ERR_IO = 5,
  GZ_ERR_CAPACITY = 6,
  GZ_ERR_UNSUPPORTED = 7
} gz_status;

typedef enum { GZ_GAME_TICTACTOE = 0, GZ_GAME_CONNECT4 = 1, GZ_GAME_CHESS = 2 } gz_game;
typedef enum { GZ_NET_GAT = 0, GZ_NET_RESNET = 1 } gz_net_kind;

/* Arithmetic of the forward pass.  AUTO: fp32 SIMT for TicTacToe, fp16
 * tensor-core operands with fp32 accumulation for the Connect4 GAT, the
 * chess GAT and the Connect4 ResNet.  FP16: fp16 tensor-core operands (11
 * significant bits, activations rounded to nearest; activations must stay
 * below 65504 in magnitude).  BF16: bf16 tensor-core operands (8 significant
 * bits, fp32 range; activations stochastically rounded), the same speed.
 * FP32: SIMT fp32 (GAT only).  gz_net_kernel_name() names the resolved
 * kernel and format. */
typedef enum { GZ_PREC_AUTO = 0, GZ_PREC_FP32 = 1, GZ_PREC_BF16 = 2, GZ_PREC_FP16 = 3 } gz_precision;

typedef struct gz_net gz_net;
typedef struct gz_mcts gz_mcts;

typedef struct {
  int game;      /* gz_game */
  int kind;      /* gz_net_kind */
  int precision; /* gz_precision */
  int max_batch; /* largest n passed to the host-buffer calls (device staging) */
} gz_net_config;

typedef struct {
  int game;               /* GZ_GAME_TICTACTOE or GZ_GAME_CONNECT4 */
  int trees;              /* concurrent games (one search tree each) */
  int leaves_per_tree;    /* leaves selected per tree per wave */
  float c_puct;           /* exploration constant */
  int virtual_loss;       /* virtual visits (value -1 each) per selection in flight */
  int node_capacity;      /* node pool per tree */
  float dirichlet_alpha;  /* root noise concentration */
  float dirichlet_eps;    /* root noise weight; 0 disables the noise */
  uint64_t seed;          /* noise and move-sampling seed */
} gz_mcts_config;

const char* gz_status_string(gz_status s);
const char* gz_last_error(void);
/* Library version string. */
const char* gz_version(void);

/* ---- games ---------------------------------------------------------------
 * Sizes of a game: nodes, rows, cols, actions, features, gat_layers,
 * policy_per_node, board_bytes, graph_nnz (9 ints).  Replaces
 * IGame::get_board_size / get_action_size (games/game.cuh:15-16). */
gz_status gz_game_shape(int game, int32_t out[9]);
/* Board-graph CSR: row_ptr[nodes+1], col[nnz]. */
gz_status gz_game_graph(int game, int32_t* row_ptr, int32_t* col);
/* IGame rules for TicTacToe / Connect4 on int8 boards (games/game.cuh:17-20;
 * connect4.cu:22-87, tictactoe.cu:24-66).
 *   gz_game_next_state: next = board with `action` played by `player`;
 *                       *next_player = -player.  GZ_ERR_INVALID_ARG if illegal.
 *   gz_game_valid_moves: valid[actions] = 1 for legal actions.
 *   gz_game_ended: *result = 1 if `player` has won, -1 if the opponent has,
 *                  2 for a draw (full board), 0 while the game continues.
 *                  (The reference returns a draw marker that its int return
 *                  type truncates to 0, connect4.cu:86.) */
gz_status gz_game_next_state(int game, const int8_t* board, int player, int action, int8_t* next_board,
                             int* next_player);
gz_status gz_game_valid_moves(int game, const int8_t* board, uint8_t* valid);
gz_status gz_game_ended(int game, const int8_t* board, int player, int* result);

/* ---- synthetic inputs (host) -------------------------------------------- */
/* Number of floats in the weight blob of (game, kind). */
size_t gz_weight_count(int game, int kind);
/* Seeded Glorot-uniform weights; bias_scale > 0 draws biases U(+-bias_scale);
 * bf16_exact != 0 rounds every value to a bfloat16-representable float. */
gz_status gz_synth_weights(int game, int kind, uint64_t seed, float bias_scale, int bf16_exact, float* out,
                           size_t n_floats);
/* n random legal non-terminal positions (uniform random playouts), indices
 * first..first+n-1 of the seeded stream.  boards [n][board_bytes], side [n].
 * Chess: k ~ U{0..120} random legal plies from the initial position, 66-byte
 * records (64 squares, castling rights, en-passant square). */
gz_status gz_synth_positions(int game, uint64_t seed, uint64_t first, int n, int8_t* boards, int8_t* side);
/* The same positions made on the device (one thread per position; byte for
 * byte what gz_synth_positions writes), into device buffers d_boards
 * [n][board_bytes] and d_side [n], on `stream` (a cudaStream_t; NULL = the
 * legacy default stream).  Asynchronous; launch errors return GZ_ERR_CUDA. */
gz_status gz_synth_positions_device(int game, uint64_t seed, uint64_t first, int n, int8_t* d_boards, int8_t* d_side,
                                    void* stream);

/* ---- chess rules (host) ---------------------------------------------------
 * Replace the move generation of games/chess/chess.cu:677-1071 (which does
 * not compile) for the position generator: a legal generator with castling,
 * en passant and promotions over the 66-byte record and side (+1 white). */
/* Number of legal moves of `side`. */
gz_status gz_chess_legal_count(const int8_t* board, int side, int* count);
/* Leaf count of the legal move tree to `depth` (0..6): the rules'
 * known-answer check against published perft counts. */
gz_status gz_chess_perft(const int8_t* board, int side, int depth, uint64_t* nodes);
/* Chess as an IGame (games/game.cuh:17-20; games/chess/chess.cu:94-135,
 * 216-282).  Actions live in the reference's space of 64 x 73 = 4672:
 * from * 73 + t, t < 64 the destination square (ordinary moves, castling as
 * the king's two-square step, promotion to a queen), t = 64 + u a straight
 * underpromotion (u = 0 knight, 1 bishop, 2 rook; the reference's
 * 64 + piece - KNIGHT), 67 + u and 70 + u underpromotions capturing toward
 * the lower and the higher file.  Every legal move has its own index.
 *   gz_chess_legal_actions: the legal moves' indices in generation order
 *                           (actions[256]), *count of them.
 *   gz_chess_valid_moves:   valid[4672] = 1 for legal actions.
 *   gz_chess_next_state:    the record after `action` and the side to move
 *                           next; GZ_ERR_INVALID_ARG if the action is illegal.
 *   gz_chess_ended:         for the side to move: 0 while it has a legal
 *                           move, -1 if checkmated, 2 for stalemate.  The
 *                           50-move rule, repetitions and insufficient
 *                           material are not tracked. */
gz_status gz_chess_legal_actions(const int8_t* board, int side, int16_t* actions, int* count);
gz_status gz_chess_valid_moves(const int8_t* board, int side, uint8_t* valid);
gz_status gz_chess_next_state(const int8_t* board, int side, int action, int8_t* next_board, int* next_side);
gz_status gz_chess_ended(const int8_t* board, int side, int* result);
/* Legal actions of n positions on the device: d_boards [n][66], d_side [n]
 * in; d_actions [n][256] (generation order, -1 after the last) and
 * d_counts [n] out, on `stream`.  The same lists as gz_chess_legal_actions. */
gz_status gz_chess_legal_actions_device(const int8_t* d_boards, const int8_t* d_side, int n, int16_t* d_actions,
                                        int32_t* d_counts, void* stream);

/* ---- network: INeuralNet replacement ------------------------------------ */
/* create_gat_model / create_resnet_model / create_neural_net
 * (networks/gat/gat.cu:681-696, networks/resnet/resnet.cu:259-272,
 * networks/neural_network.c:6-13). */
gz_status gz_net_create(const gz_net_config* cfg, int device, gz_net** out);
/* INeuralNet::destroy (neural_network.h:25). */
gz_status gz_net_destroy(gz_net* net);
size_t gz_net_weight_count(const gz_net* net);
/* Name of the forward kernel and operand format this handle uses:
 * "gat_tc_fp16", "gat_tc_bf16", "gat_simt_fp32", "resnet_tc_fp16" or
 * "resnet_tc_bf16". */
const char* gz_net_kernel_name(const gz_net* net);
/* Weights as one fp32 blob in the documented layout (the replacement for the
 * reference's per-tensor cudaMalloc + cuRAND init, gat.cu:720-789). */
gz_status gz_net_load_weights(gz_net* net, const float* host_blob, size_t n_floats);
gz_status gz_net_save_weights(const gz_net* net, float* host_blob, size_t n_floats);
/* INeuralNet::predict over a batch, all pointers on the device of `net`:
 * boards [n][board_bytes], side [n], pi [n][actions], v [n]. */
gz_status gz_net_predict_batch(gz_net* net, const int8_t* d_boards, const int8_t* d_side, int n, float* d_pi,
                               float* d_v, void* stream);
/* Synchronises and reports GZ_ERR_TIMEOUT if a bounded wait inside a forward
 * kernel gave up since the last check (the word is then cleared). */
gz_status gz_net_check(gz_net* net);
/* Same with host buffers: copies in, evaluates, copies out, synchronises.
 * n <= max_batch.  Page-locked caller buffers (cudaHostAlloc /
 * cudaHostRegister) are transferred directly, pageable ones through the
 * net's page-locked staging; a chess call of n >= 1024 runs as four pieces
 * whose transfers and host copies overlap the next piece's forward pass
 * (same results).  Other games read page-locked buffers that are mapped
 * into the device's address space (cudaHostAlloc'd memory is) straight
 * from the forward kernel, which also writes the outputs there. */
gz_status gz_net_predict_host(gz_net* net, const int8_t* h_boards, const int8_t* h_side, int n, float* h_pi,
                              float* h_v);
/* INeuralNet::predict (neural_network.h:22): one position given as the
 * canonical float board (own stones +1, opponent -1; the reference's
 * get_canonical_form, connect4.cu:89-93), host pointers. */
gz_status gz_net_predict(gz_net* net, const float* h_board, float* h_pi, float* h_v);
/* INeuralNet::save_checkpoint / load_checkpoint (neural_network.h:23-24; the
 * reference writes a libtorch archive, networks/gat/gat.cu:201-337).  File:
 * "GZB200W1" magic, then int32 version, game, kind, reserved, uint64 count,
 * count fp32 weights (little endian, the weight-blob layout), uint64 FNV-1a
 * hash of the weight bytes.  Load checks game, kind, count and hash
 * (GZ_ERR_IO on any mismatch or short file). */
gz_status gz_net_save_checkpoint(const gz_net* net, const char* path);
gz_status gz_net_load_checkpoint(gz_net* net, const char* path);
/* INeuralNet::broadcast_weights (neural_network.h:27): ncclBroadcast of the
 * weight blob from `root` over an existing communicator (ncclComm_t). */
gz_status gz_net_broadcast(gz_net* net, void* nccl_comm, int root, void* stream);

/* ---- NCCL bootstrap without MPI (the reference uses MPI_Bcast of the id,
 * main.cu:59-61) ---------------------------------------------------------- */
/* 128-byte ncclUniqueId. */
gz_status gz_nccl_unique_id(uint8_t out[128]);
gz_status gz_nccl_comm_init(const uint8_t id[128], int world, int rank, int device, void** comm);
gz_status gz_nccl_comm_destroy(void* comm);

/* ---- batched PUCT search (mcts/mcts.cu, self_play/self_play.cu:610-758) --
 * Every game: TicTacToe and Connect4 boards of `nodes` bytes; chess
 * 66-byte records with actions in the 64 x 73 space of gz_chess_valid_moves
 * (root statistics [trees][4672]; a node reached by checkmate is a loss for
 * its player to move, stalemate a draw; a finished game restarts from the
 * initial position).  A chess pool reserves 64 edges per node (about 35 are
 * used on average; gz_mcts_check reports an overflow).  Self-play and the
 * arena play TicTacToe and Connect4 (GZ_ERR_UNSUPPORTED for chess). */
gz_status gz_mcts_create(const gz_mcts_config* cfg, int device, gz_mcts** out);
gz_status gz_mcts_destroy(gz_mcts* m);
/* Root positions, device arrays boards [trees][board bytes], side [trees]
 * (replaces mcts_init, mcts/mcts.cu:10). */
gz_status gz_mcts_reset_roots(gz_mcts* m, const int8_t* d_boards, const int8_t* d_side, void* stream);
/* One selection pass; fills the leaf batch (trees * leaves_per_tree). */
gz_status gz_mcts_select(gz_mcts* m, void* stream);
/* Device pointers of the leaf batch: boards [L][nodes], side [L], terminal [L]. */
gz_status gz_mcts_leaf_buffers(gz_mcts* m, int8_t** d_boards, int8_t** d_side, int8_t** d_terminal);
/* Copies the leaf batch to host buffers and synchronises (for callers that
 * evaluate leaves themselves); any pointer may be NULL. */
gz_status gz_mcts_copy_leaves(gz_mcts* m, int8_t* h_boards, int8_t* h_side, int8_t* h_terminal, void* stream);
/* Backup of the current wave with the leaves' evaluations (device arrays
 * pi [L][actions], v [L]). */
gz_status gz_mcts_backup(gz_mcts* m, const float* d_pi, const float* d_v, void* stream);
/* select -> net evaluation of the leaf batch -> backup. */
gz_status gz_mcts_step(gz_mcts* m, gz_net* net, void* stream);
/* Waves until every tree has run `sims` more simulations (mcts_run_batch,
 * mcts/mcts.cu:221-263). */
gz_status gz_mcts_run(gz_mcts* m, gz_net* net, int sims, void* stream);
/* Root visit counts [trees][actions] (and optionally value sums) to host;
 * synchronises and reports any capacity error of earlier kernels. */
gz_status gz_mcts_root_stats(gz_mcts* m, int32_t* h_visits, float* h_wsum, void* stream);
/* Node and edge pool use per tree, to host. */
gz_status gz_mcts_tree_sizes(gz_mcts* m, int32_t* h_nodes, int32_t* h_edges, void* stream);
/* Actions from root visits (mcts_select_action, mcts/mcts.cu:40-66): sampled
 * in proportion to N for the first temp_moves moves of a game, then argmax.
 * d_actions [trees]. */
gz_status gz_mcts_choose(gz_mcts* m, int temp_moves, int32_t* d_actions, void* stream);
/* Advance roots (mcts_update_with_move, mcts/mcts.cu:68-103); a subtree is
 * kept while `reserve` pool nodes remain.  d_done [trees] (may be NULL). */
gz_status gz_mcts_play(gz_mcts* m, const int32_t* d_actions, int reserve, int8_t* d_done, void* stream);
/* Sticky device error of the search kernels (0 none, 1 node pool, 2 edge
 * pool, 3 depth); synchronises. */
gz_status gz_mcts_check(gz_mcts* m);

/* ---- self-play episodes and training examples (self_play/self_play.cu) --- */
#define GZ_EXAMPLE_CELLS 64 /* MAX_BOARD_SIZE, games/game.cuh:7 */
/* TrainingExample of self_play/self_play.cuh:56-60 (516 bytes, no padding):
 * the record the reference's train_examples_*.bin files hold.  board is the
 * canonical position (board x player to move, connect4.cu:89-93), pi the
 * search policy over actions, v the game's outcome for the player to move
 * (+1 win, -1 loss, 0 draw); unused cells are zero. */
typedef struct gz_train_example {
  int32_t board[GZ_EXAMPLE_CELLS];
  float pi[GZ_EXAMPLE_CELLS];
  float v;
} gz_train_example;
typedef struct gz_selfplay gz_selfplay;
/* Self-play state on top of a search handle (which it uses, not owns):
 * per-tree logs of the game in progress and a device buffer for up to
 * max_examples finished examples (replaces SelfPlayPipeline's d_examples,
 * self_play.cu:102-105). */
gz_status gz_selfplay_create(gz_mcts* m, int max_examples, gz_selfplay** out);
gz_status gz_selfplay_destroy(gz_selfplay* sp);
/* Plays moves on every tree until n_games more games have ended
 * (execute_self_play / parallel_self_play_kernel, self_play.cu:75-145,
 * 403-472): per move `sims` simulations, the root recorded as an example
 * with pi = N / sum N for the first temp_moves moves of a game and one-hot
 * on the most visited move afterwards (mcts_get_policy, 645-662), a move
 * chosen as gz_mcts_choose does, the roots advanced (a finished game's tree
 * starts a new game).  Ended games' examples go to the buffer in the order
 * the games ended (ties: tree order).  Synchronises once per move.
 * GZ_ERR_CAPACITY when the buffer overflows: it then holds the games that
 * ended before the first one that did not fit, the rest of that move's
 * ended games are lost (gz_selfplay_take empties the buffer). */
gz_status gz_selfplay_run(gz_selfplay* sp, gz_net* net, int n_games, int sims, int temp_moves, void* stream);
/* Copies the buffered examples to the host, in order, and empties the
 * buffer; *n_examples and *n_games (either may be NULL) receive the counts.
 * GZ_ERR_CAPACITY (nothing copied, buffer kept) if capacity is too small. */
gz_status gz_selfplay_take(gz_selfplay* sp, gz_train_example* h_out, int64_t capacity, int64_t* n_examples,
                           int64_t* n_games);
/* Arena (arena/arena.cu:31-106 play_game / play_games, used by
 * pit_against_previous_version, self_play.cu:576-606): n_games games of
 * net_a against net_b, played up to one game per tree of `m` at a time.
 * Every move is searched from a fresh root with `sims` simulations by the
 * network of the side to move, which plays its most visited move (the
 * reference's NNet player, players/players.cu:96-104).  Net A moves first in
 * the first n_games / 2 games, net B in the rest (the reference swaps the
 * players half way, arena.cu:98-102).  Results count games won by each
 * network and draws.  For a deterministic arena create `m` without root
 * noise (dirichlet_eps 0); its trees are overwritten. */
gz_status gz_arena_play(gz_mcts* m, gz_net* net_a, gz_net* net_b, int n_games, int sims, int32_t* a_wins,
                        int32_t* b_wins, int32_t* draws, void* stream);
/* save_train_examples (self_play.cu:510-534): the reference's file layout,
 * int32 number of iterations, then per iteration int32 count and count
 * 516-byte records (little endian).  iters[i] holds counts[i] examples. */
gz_status gz_train_examples_save(const char* path, int n_iters, const gz_train_example* const* iters,
                                 const int32_t* counts);
/* load_train_examples (self_play.cu:536-573): reads such a file.  With
 * out == NULL only *n_iters and *total are set (sizes for a second call);
 * otherwise the iterations' records go to `out` back to back and counts[i]
 * gets iteration i's count (max_iters entries).  GZ_ERR_IO on a short or
 * malformed file, GZ_ERR_CAPACITY if capacity or max_iters is too small. */
gz_status gz_train_examples_load(const char* path, gz_train_example* out, int64_t capacity, int32_t* counts,
                                 int max_iters, int* n_iters, int64_t* total);

/* ---- training (GAT nets and the Connect4 ResNet) ---------------------------
 * Loss per position: -sum_a pi_a log p_a + (z - v)^2, averaged over the
 * batch (the reference's loss gradients, networks/gat/gat.cu:1040-1109:
 * softmax cross-entropy p - pi, value MSE 2 (v - z); the ResNet's losses
 * at networks/resnet/resnet.cu:669-699 are the same two terms).  fp32
 * forward and backward on CUDA cores, every reduction in a fixed order (a
 * step is reproducible bit for bit), then Adam as torch::optim::Adam with
 * weight decay added to the gradient (gat.cu:71).  The ResNet trains with
 * its BN in inference form, as gz_net_predict evaluates it: BN scales and
 * shifts are trained, the stored means and variances get a zero gradient
 * and are not updated.  After every step the net's tensor-core weights are
 * repacked, so predictions use the new weights. */
typedef struct {
  float learning_rate; /* 1e-3 (gat.cu:712) */
  float weight_decay;  /* 1e-4 (gat.cu:713) */
  float beta1, beta2;  /* 0.9, 0.999 */
  float eps;           /* 1e-8 */
  int batch_size;      /* positions per rank per step, 64 (gat.cu:716) */
  int epochs;          /* 10 (gat.cu:717) */
  uint64_t seed;       /* example order: a fresh permutation per epoch */
} gz_train_config;
typedef struct {
  float policy_loss; /* mean over the last epoch's steps (this rank's batches) */
  float value_loss;
  int64_t steps;     /* optimizer steps taken by the net so far */
} gz_train_stats;
/* The reference's defaults (gat.cu:702-718 init_model_config). */
void gz_train_config_default(gz_train_config* cfg);
/* Loss and gradient of one batch, no update: device boards [n][board bytes],
 * side [n], target policies pi [n][actions], target values v [n].  The
 * gradient (gz_net_weight_count floats, the weight blob's layout) goes to
 * d_grad when it is not NULL, the two loss terms to h_loss (policy, value)
 * when it is not NULL.  GAT nets of every game and the Connect4 ResNet.
 * Synchronises. */
gz_status gz_net_loss_grad(gz_net* net, const int8_t* d_boards, const int8_t* d_side, const float* d_pi,
                           const float* d_v, int n, float* d_grad, float h_loss[2], void* stream);
/* One optimizer step on one batch (device buffers as above).  With a
 * communicator (ncclComm_t, world > 1) every rank passes its own batch: the
 * gradient buckets (one per layer, one for the heads) are all-reduced on a
 * side stream as the backward pass completes them, averaged, and every rank
 * applies the same update (INeuralNet::train_distributed, gat.cu:381-543,
 * whose gradient all-reduce is at 496-514).  h_loss (may be NULL) gets this
 * rank's two loss terms.  Synchronises. */
gz_status gz_net_train_step(gz_net* net, const int8_t* d_boards, const int8_t* d_side, const float* d_pi,
                            const float* d_v, int n, const gz_train_config* cfg, void* nccl_comm, int world,
                            float h_loss[2], void* stream);
/* INeuralNet::train (gat.cu:82-148): `epochs` passes over n host examples
 * (canonical boards as self-play writes them; TicTacToe and Connect4), each
 * pass in a fresh seeded order, floor(n / (batch_size * world)) steps per
 * pass, the last partial batch dropped as in the reference.  With a
 * communicator every rank must hold the same examples: step k of a pass
 * gives rank r the r-th batch_size slice of the k-th batch_size * world
 * block of the order.  stats may be NULL. */
gz_status gz_net_train(gz_net* net, const gz_train_example* examples, int64_t n, const gz_train_config* cfg,
                       void* nccl_comm, int rank, int world, gz_train_stats* stats);
/* The positions of step `step` of pass `epoch` that rank `rank` trains on
 * (gz_net_train's order), as example indices into out[batch_size]; host
 * only, for callers that stage their own batches. */
gz_status gz_train_batch_indices(int64_t n, const gz_train_config* cfg, int epoch, int64_t step, int rank, int world,
                                 int64_t* out);
/* Gradient bucket k of a GAT net of `game` (k < layers: layer k's W, b and a;
 * k == layers: the policy and value heads), as an offset and a length in
 * floats of the weight layout; gz_net_train_step all-reduces the buckets
 * from the heads down to layer 0, each as soon as the backward pass has
 * produced it.  (The ResNet's 12 buckets, in the order they complete: the
 * heads, blocks 9 down to 0, the stem.)  Host only. */
gz_status gz_train_bucket_range(int game, int k, size_t* offset, size_t* count);

/* ---- allocation-free leaf evaluation --------------------------------------
 * No counterpart in the reference.  For callers that may not allocate device
 * memory (a plugin inside a host application that fixes the device-memory
 * budget at start-up; a latency-critical loop that cannot pay for
 * cudaMalloc/cudaFree, which synchronise the device): Connect4 GAT leaf
 * evaluation (the tensor-core kernel and operand format of a net created with
 * GZ_PREC_AUTO) from host weights (the Connect4 GAT blob), host positions
 * int8 [n][42] + side [n], into host pi [n][7], v [n].
 * It calls no cudaMalloc/cudaFree: all device staging lives in one static
 * device array of gz_gat_c4_noalloc_scratch_bytes() (about 2.3 MB), reserved
 * on every GPU that loads the library until the process exits.  n is limited
 * to gz_gat_c4_noalloc_max_batch() (4096); larger n returns
 * GZ_ERR_INVALID_ARG.  The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress) with that device current, so make that first
 * call before any stream capture; after a cudaDeviceReset the next call looks
 * it up again.  All calls share the array: calls that overlap in time on one
 * device race and must be serialised by the caller.  Every call uploads the
 * 1.4 MB weight blob and repacks it before the forward pass, on the device's
 * legacy default stream (which waits for the process's blocking streams).
 * Synchronous (returns when the outputs are in host memory). */
gz_status gz_gat_c4_predict_noalloc(int device, const float* h_weights, size_t n_weights, const int8_t* h_boards,
                                    const int8_t* h_side, int n, float* h_pi, float* h_v);
size_t gz_gat_c4_noalloc_scratch_bytes(void);
int gz_gat_c4_noalloc_max_batch(void);

/* ---- failure detection ---------------------------------------------------
 * Runs, on `device`, a one-block kernel whose thread waits on an mbarrier
 * that nothing ever arrives at, through the same bounded wait every kernel of
 * this library uses, with a limit of `limit_us`.  Returns GZ_ERR_TIMEOUT when
 * the wait gave up and the kernel exited cleanly (the expected outcome),
 * GZ_OK if it somehow completed, GZ_ERR_CUDA on a launch error.  The CUDA
 * context stays usable afterwards. */
gz_status gz_selftest_wait_timeout(int device, int limit_us);

#ifdef __cplusplus
}
#endif

#endif /* GRAPHZERO_B200_H */
