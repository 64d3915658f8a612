// Seeded synthetic inputs: network weights and random legal positions.
//
// The reference seeds cuRAND with time(NULL) (networks/gat/gat.cu:769,
// networks/resnet/resnet.cu:396-431), so its weights are not reproducible;
// here every weight and position is a pure function of (seed, index), so any
// shard of a batch can be regenerated on any rank or process.
//
// The position generators (make_position, chess::make_position) compile for
// host and device alike and give identical positions on both; the weight
// generators are host code.
#pragma once
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "gz_games.h"

namespace gz {

// splitmix64 (Steele, Lea, Flood 2014).
struct SplitMix {
  uint64_t s;
  GZ_HDI explicit SplitMix(uint64_t seed) : s(seed) {}
  GZ_HDI uint64_t next() {
    uint64_t z = (s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
  }
  // Uniform in [0, 1) with 24 random bits.
  GZ_HDI float uniform() { return (float)(next() >> 40) * (1.0f / 16777216.0f); }
  // Uniform integer in [0, n).
  GZ_HDI uint32_t below(uint32_t n) { return (uint32_t)(((next() >> 32) * (uint64_t)n) >> 32); }
  // Standard normal (Box-Muller on two uniforms in (0, 1]).
  float normal() {
    double u1 = ((double)(next() >> 11) + 1.0) * (1.0 / 9007199254740992.0);
    double u2 = (double)(next() >> 11) * (1.0 / 9007199254740992.0);
    return (float)(sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2));
  }
};

GZ_HDI uint64_t mix_seed(uint64_t seed, uint64_t stream) {
  SplitMix m(seed ^ (stream * 0xD1B54A32D192ED03ull));
  return m.next();
}

// Round-to-nearest-even to the nearest bfloat16 value, returned as fp32.
inline float round_to_bf16(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7F800000u) == 0x7F800000u) return x;  // inf / nan unchanged
  u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
  float y;
  memcpy(&y, &u, 4);
  return y;
}

// Weight generation options.
struct WeightOpts {
  float bias_scale = 0.0f;  // biases ~ U(-bias_scale, bias_scale); 0 = zero biases
  bool bf16_exact = true;   // round every weight to a bfloat16-representable value
};

inline void fill_glorot(SplitMix& r, float* w, size_t n, int fan_in, int fan_out, const WeightOpts& o) {
  float lim = sqrtf(6.0f / (float)(fan_in + fan_out));
  for (size_t i = 0; i < n; ++i) {
    float v = (2.0f * r.uniform() - 1.0f) * lim;
    w[i] = o.bf16_exact ? round_to_bf16(v) : v;
  }
}

inline void fill_bias(SplitMix& r, float* w, size_t n, const WeightOpts& o) {
  for (size_t i = 0; i < n; ++i) {
    float v = o.bias_scale == 0.0f ? 0.0f : (2.0f * r.uniform() - 1.0f) * o.bias_scale;
    w[i] = o.bf16_exact ? round_to_bf16(v) : v;
  }
}

// GAT weights, Glorot-uniform U(+-sqrt(6 / (fan_in + fan_out))).
inline void make_gat_weights(int game, uint64_t seed, const WeightOpts& o, float* out) {
  GatLayout t = gat_layout(game);
  SplitMix r(mix_seed(seed, 0x6A7));
  for (int l = 0; l < t.L; ++l) {
    int fin = l == 0 ? t.F : kHidden;
    fill_glorot(r, out + t.W[l], (size_t)fin * kHidden, fin, kHidden, o);
    fill_bias(r, out + t.b[l], kHidden, o);
    fill_glorot(r, out + t.a[l], kHeads * 2 * kHeadDim, 2 * kHeadDim, 1, o);
  }
  fill_glorot(r, out + t.w_pi, (size_t)kHidden * t.P, kHidden, t.P, o);
  fill_bias(r, out + t.b_pi, t.P, o);
  fill_glorot(r, out + t.W_v1, (size_t)kHidden * kValueHidden, kHidden, kValueHidden, o);
  fill_bias(r, out + t.b_v1, kValueHidden, o);
  fill_glorot(r, out + t.w_v2, kValueHidden, kValueHidden, 1, o);
  fill_bias(r, out + t.b_v2, 1, o);
}

// BN parameters: gamma ~ U(0.8, 1.2), beta ~ N(0, 0.1), mean ~ N(0, 0.1),
// var ~ U(0.5, 1.5).
inline void fill_bn(SplitMix& r, float* bn, int C, const WeightOpts& o) {
  for (int c = 0; c < C; ++c) bn[c] = 0.8f + 0.4f * r.uniform();
  for (int c = 0; c < C; ++c) bn[C + c] = 0.1f * r.normal();
  for (int c = 0; c < C; ++c) bn[2 * C + c] = 0.1f * r.normal();
  for (int c = 0; c < C; ++c) bn[3 * C + c] = 0.5f + r.uniform();
  if (o.bf16_exact)
    for (int i = 0; i < 4 * C; ++i) bn[i] = round_to_bf16(bn[i]);
}

// Connect4 ResNet weights (He-style Glorot on conv fans, BN as above).
inline void make_resnet_weights(uint64_t seed, const WeightOpts& o, float* out) {
  ResLayout t = res_layout();
  const int C = kResChannels;
  SplitMix r(mix_seed(seed, 0x5E5));
  fill_glorot(r, out + t.stem_w, (size_t)C * 9 * kResInPlanes, 9 * kResInPlanes, 9 * C, o);
  fill_bn(r, out + t.stem_bn, C, o);
  for (int k = 0; k < kResBlocks; ++k) {
    fill_glorot(r, out + t.conv1_w[k], (size_t)C * 9 * C, 9 * C, 9 * C, o);
    fill_bn(r, out + t.bn1[k], C, o);
    fill_glorot(r, out + t.conv2_w[k], (size_t)C * 9 * C, 9 * C, 9 * C, o);
    fill_bn(r, out + t.bn2[k], C, o);
  }
  fill_glorot(r, out + t.pol_w, 2 * C, C, 2, o);
  fill_bn(r, out + t.pol_bn, 2, o);
  fill_glorot(r, out + t.pol_fc, 84 * 7, 84, 7, o);
  fill_bias(r, out + t.pol_fc_b, 7, o);
  fill_glorot(r, out + t.val_w, C, C, 1, o);
  fill_bn(r, out + t.val_bn, 1, o);
  fill_glorot(r, out + t.val_fc1, 42 * kResValueHidden, 42, kResValueHidden, o);
  fill_bias(r, out + t.val_fc1_b, kResValueHidden, o);
  fill_glorot(r, out + t.val_fc2, kResValueHidden, kResValueHidden, 1, o);
  fill_bias(r, out + t.val_fc2_b, 1, o);
}

// Random legal TicTacToe / Connect4 position: k ~ U{0..max_plies} uniformly
// random legal moves from the empty board; a move that would end the game is
// not played and the playout stops there, so every position is non-terminal.
// Writes board[N] and returns the side to move (+1 first player, -1 second).
GZ_HDI int make_position(int game, uint64_t seed, uint64_t index, int8_t* board) {
  GameShape s = game_shape(game);
  SplitMix r(mix_seed(seed, 0x9051 + index));
  memset(board, 0, (size_t)s.board_bytes);
  int max_plies = s.nodes - 1;  // 8 (TicTacToe), 41 (Connect4)
  int k = (int)r.below((uint32_t)max_plies + 1);
  int side = 1;
  for (int ply = 0; ply < k; ++ply) {
    int legal[9], n = 0;
    for (int a = 0; a < s.actions; ++a)
      if (action_legal(game, board, a)) legal[n++] = a;
    if (n == 0) break;
    int a = legal[r.below((uint32_t)n)];
    int8_t trial[64];
    memcpy(trial, board, (size_t)s.nodes);
    int sq = apply_action(game, trial, a, side);
    if (outcome_after(game, trial, sq, side) != 0) break;
    memcpy(board, trial, (size_t)s.nodes);
    side = -side;
  }
  return side;
}

}  // namespace gz
