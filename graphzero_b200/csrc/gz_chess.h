// Chess rules for the position generator (host code): legal move
// generation, move application, perft, and random legal playouts.
//
// Record layout (66 bytes, the network's input): squares 0..63 = rank * 8 +
// file (a1 = 0, h8 = 63), piece codes +1..+6 = white P N B R Q K and
// -1..-6 = black (games/chess/chess.cuh:11-21); byte 64 castling rights
// (bit 0 white king side, 1 white queen side, 2 black king side, 3 black
// queen side); byte 65 the en-passant target square (the square a pawn that
// just advanced two ranks passed over) or -1.  The side to move travels
// beside the record (+1 white, -1 black).
//
// The reference's own move generator (games/chess/chess.cu:677-1071) does
// not compile; this is a standard legal generator: pseudo-legal moves,
// then the ones that leave the mover's king attacked are dropped; castling
// needs the rook on its corner, empty squares between, and the king's
// start, transit and destination squares unattacked.  The 50-move rule and
// repetitions are not tracked (positions are network inputs).
#pragma once
#include <stdint.h>
#include <string.h>

#include "gz_synth.h"

namespace gz {
namespace chess {

enum Piece : int { kPawn = 1, kKnight = 2, kBishop = 3, kRook = 4, kQueen = 5, kKing = 6 };

struct Pos {
  int8_t sq[64];
  uint8_t castle;  // bits: 0 WK, 1 WQ, 2 BK, 3 BQ
  int8_t ep;       // en-passant target square or -1
  int8_t side;     // +1 white to move, -1 black
};

struct Move {
  int8_t from, to, promo;  // promo: 0 or the promoted piece type (unsigned)
};

inline int file_of(int s) { return s & 7; }
inline int rank_of(int s) { return s >> 3; }
inline int sgn(int v) { return (v > 0) - (v < 0); }

inline void start_pos(Pos& p) {
  static const int8_t back[8] = {kRook, kKnight, kBishop, kQueen, kKing, kBishop, kKnight, kRook};
  memset(p.sq, 0, 64);
  for (int f = 0; f < 8; ++f) {
    p.sq[f] = back[f];
    p.sq[8 + f] = kPawn;
    p.sq[48 + f] = -kPawn;
    p.sq[56 + f] = (int8_t)-back[f];
  }
  p.castle = 0xF;
  p.ep = -1;
  p.side = 1;
}

inline void to_record(const Pos& p, int8_t* rec) {
  memcpy(rec, p.sq, 64);
  rec[64] = (int8_t)p.castle;
  rec[65] = p.ep;
}

inline void from_record(const int8_t* rec, int side, Pos& p) {
  memcpy(p.sq, rec, 64);
  p.castle = (uint8_t)rec[64] & 0xF;
  p.ep = rec[65];
  p.side = (int8_t)(side >= 0 ? 1 : -1);
}

// Offsets as (file, rank) steps.
constexpr int kKnightD[8][2] = {{1, 2}, {2, 1}, {2, -1}, {1, -2}, {-1, -2}, {-2, -1}, {-2, 1}, {-1, 2}};
constexpr int kKingD[8][2] = {{1, 0}, {1, 1}, {0, 1}, {-1, 1}, {-1, 0}, {-1, -1}, {0, -1}, {1, -1}};
constexpr int kDiagD[4][2] = {{1, 1}, {-1, 1}, {-1, -1}, {1, -1}};
constexpr int kLineD[4][2] = {{1, 0}, {0, 1}, {-1, 0}, {0, -1}};

inline bool on_board(int f, int r) { return (unsigned)f < 8u && (unsigned)r < 8u; }

// Is square s attacked by side `by` (+1 / -1)?
inline bool attacked(const Pos& p, int s, int by) {
  const int f = file_of(s), r = rank_of(s);
  // pawns of `by` attack diagonally forward (rank + by)
  for (int df = -1; df <= 1; df += 2) {
    const int pf = f + df, pr = r - by;
    if (on_board(pf, pr) && p.sq[pr * 8 + pf] == by * kPawn) return true;
  }
  for (auto& d : kKnightD) {
    const int nf = f + d[0], nr = r + d[1];
    if (on_board(nf, nr) && p.sq[nr * 8 + nf] == by * kKnight) return true;
  }
  for (auto& d : kKingD) {
    const int nf = f + d[0], nr = r + d[1];
    if (on_board(nf, nr) && p.sq[nr * 8 + nf] == by * kKing) return true;
  }
  for (auto& d : kDiagD)
    for (int nf = f + d[0], nr = r + d[1]; on_board(nf, nr); nf += d[0], nr += d[1]) {
      const int v = p.sq[nr * 8 + nf];
      if (v == 0) continue;
      if (v == by * kBishop || v == by * kQueen) return true;
      break;
    }
  for (auto& d : kLineD)
    for (int nf = f + d[0], nr = r + d[1]; on_board(nf, nr); nf += d[0], nr += d[1]) {
      const int v = p.sq[nr * 8 + nf];
      if (v == 0) continue;
      if (v == by * kRook || v == by * kQueen) return true;
      break;
    }
  return false;
}

inline int king_square(const Pos& p, int side) {
  for (int s = 0; s < 64; ++s)
    if (p.sq[s] == side * kKing) return s;
  return -1;
}

// Apply a (pseudo-)legal move in place.
inline void apply(Pos& p, const Move& m) {
  const int me = p.side, v = p.sq[m.from], type = v * me;
  const int ep_capture = (type == kPawn && m.to == p.ep && p.sq[m.to] == 0) ? m.to - 8 * me : -1;
  p.sq[m.to] = m.promo ? (int8_t)(me * m.promo) : (int8_t)v;
  p.sq[m.from] = 0;
  if (ep_capture >= 0) p.sq[ep_capture] = 0;
  if (type == kKing && (m.to - m.from == 2 || m.from - m.to == 2)) {  // castling: move the rook
    const int r0 = rank_of(m.from) * 8;
    if (m.to > m.from) {
      p.sq[r0 + 5] = p.sq[r0 + 7];
      p.sq[r0 + 7] = 0;
    } else {
      p.sq[r0 + 3] = p.sq[r0 + 0];
      p.sq[r0 + 0] = 0;
    }
  }
  // castling rights: a king move clears its side's rights; anything leaving
  // or landing on a rook corner clears that corner's right
  if (type == kKing) p.castle &= me > 0 ? ~0x3u : ~0xCu;
  for (int s : {(int)m.from, (int)m.to}) {
    if (s == 7) p.castle &= ~0x1u;
    if (s == 0) p.castle &= ~0x2u;
    if (s == 63) p.castle &= ~0x4u;
    if (s == 56) p.castle &= ~0x8u;
  }
  p.ep = (type == kPawn && (m.to - m.from == 16 || m.from - m.to == 16)) ? (int8_t)((m.from + m.to) / 2) : (int8_t)-1;
  p.side = (int8_t)-me;
}

// Pseudo-legal moves of the side to move; returns the count (<= 256).
inline int pseudo_moves(const Pos& p, Move* out) {
  const int me = p.side;
  int n = 0;
  auto add = [&](int from, int to, int promo) { out[n++] = Move{(int8_t)from, (int8_t)to, (int8_t)promo}; };
  auto add_pawn = [&](int from, int to) {
    const int last = me > 0 ? 7 : 0;
    if (rank_of(to) == last)
      for (int pr : {kQueen, kRook, kBishop, kKnight}) add(from, to, pr);
    else
      add(from, to, 0);
  };
  for (int s = 0; s < 64; ++s) {
    const int v = p.sq[s];
    if (v == 0 || sgn(v) != me) continue;
    const int type = v * me, f = file_of(s), r = rank_of(s);
    if (type == kPawn) {
      const int r1 = r + me;
      if (!on_board(f, r1)) continue;
      if (p.sq[r1 * 8 + f] == 0) {
        add_pawn(s, r1 * 8 + f);
        const int start = me > 0 ? 1 : 6, r2 = r + 2 * me;
        if (r == start && p.sq[r2 * 8 + f] == 0) add(s, r2 * 8 + f, 0);
      }
      for (int df = -1; df <= 1; df += 2) {
        const int cf = f + df;
        if (!on_board(cf, r1)) continue;
        const int t = r1 * 8 + cf, tv = p.sq[t];
        if ((tv != 0 && sgn(tv) == -me) || t == p.ep) add_pawn(s, t);
      }
    } else if (type == kKnight || type == kKing) {
      const auto& D = type == kKnight ? kKnightD : kKingD;
      for (auto& d : D) {
        const int nf = f + d[0], nr = r + d[1];
        if (!on_board(nf, nr)) continue;
        const int tv = p.sq[nr * 8 + nf];
        if (tv == 0 || sgn(tv) == -me) add(s, nr * 8 + nf, 0);
      }
      if (type == kKing) {
        const int home = me > 0 ? 4 : 60, ks = me > 0 ? 0x1 : 0x4, qs = me > 0 ? 0x2 : 0x8;
        if (s == home && !attacked(p, s, -me)) {
          if ((p.castle & ks) && p.sq[s + 3] == me * kRook && p.sq[s + 1] == 0 && p.sq[s + 2] == 0 &&
              !attacked(p, s + 1, -me) && !attacked(p, s + 2, -me))
            add(s, s + 2, 0);
          if ((p.castle & qs) && p.sq[s - 4] == me * kRook && p.sq[s - 1] == 0 && p.sq[s - 2] == 0 &&
              p.sq[s - 3] == 0 && !attacked(p, s - 1, -me) && !attacked(p, s - 2, -me))
            add(s, s - 2, 0);
        }
      }
    } else {
      const bool diag = type == kBishop || type == kQueen, line = type == kRook || type == kQueen;
      for (int k = 0; k < 8; ++k) {
        if (k < 4 ? !diag : !line) continue;
        const int* d = k < 4 ? kDiagD[k] : kLineD[k - 4];
        for (int nf = f + d[0], nr = r + d[1]; on_board(nf, nr); nf += d[0], nr += d[1]) {
          const int tv = p.sq[nr * 8 + nf];
          if (tv != 0 && sgn(tv) == me) break;
          add(s, nr * 8 + nf, 0);
          if (tv != 0) break;
        }
      }
    }
  }
  return n;
}

// Legal moves of the side to move; returns the count (<= 256).
inline int legal_moves(const Pos& p, Move* out) {
  Move ps[256];
  const int np = pseudo_moves(p, ps);
  int n = 0;
  for (int i = 0; i < np; ++i) {
    Pos q = p;
    apply(q, ps[i]);
    const int k = king_square(q, p.side);
    if (k >= 0 && !attacked(q, k, -p.side)) out[n++] = ps[i];
  }
  return n;
}

inline uint64_t perft(const Pos& p, int depth) {
  if (depth == 0) return 1;
  Move ms[256];
  const int n = legal_moves(p, ms);
  if (depth == 1) return (uint64_t)n;
  uint64_t total = 0;
  for (int i = 0; i < n; ++i) {
    Pos q = p;
    apply(q, ms[i]);
    total += perft(q, depth - 1);
  }
  return total;
}

// Random legal chess position: k ~ U{0..120} uniformly random legal moves
// from the initial position; a move after which the opponent has no legal
// move (mate or stalemate) is not played and the playout stops there, so
// every position has a legal move.  Writes the 66-byte record and returns
// the side to move.
inline int make_position(uint64_t seed, uint64_t index, int8_t* rec) {
  SplitMix r(mix_seed(seed, 0xC4E55 + index));
  Pos p;
  start_pos(p);
  const int k = (int)r.below(121u);
  Move ms[256], reply[256];
  for (int ply = 0; ply < k; ++ply) {
    const int n = legal_moves(p, ms);
    if (n == 0) break;
    Pos q = p;
    apply(q, ms[r.below((uint32_t)n)]);
    if (legal_moves(q, reply) == 0) break;
    p = q;
  }
  to_record(p, rec);
  return p.side;
}

}  // namespace chess
}  // namespace gz
