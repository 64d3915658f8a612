// Chess rules: legal move generation, move application, the reference's
// action indices, game end, perft and random legal playouts.  Everything but
// perft compiles for host and device alike (GZ_HDI) and behaves identically
// on both.
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

GZ_HDI int file_of(int s) { return s & 7; }
GZ_HDI int rank_of(int s) { return s >> 3; }
GZ_HDI int sgn(int v) { return (v > 0) - (v < 0); }

GZ_HDI void start_pos(Pos& p) {
  const int8_t back[8] = {kRook, kKnight, kBishop, kQueen, kKing, kBishop, kKnight, kRook};
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

GZ_HDI void to_record(const Pos& p, int8_t* rec) {
  memcpy(rec, p.sq, 64);
  rec[64] = (int8_t)p.castle;
  rec[65] = p.ep;
}

GZ_HDI void from_record(const int8_t* rec, int side, Pos& p) {
  memcpy(p.sq, rec, 64);
  p.castle = (uint8_t)rec[64] & 0xF;
  p.ep = rec[65];
  p.side = (int8_t)(side >= 0 ? 1 : -1);
}

// Step k of each piece as (file, rank) offsets: knights and kings k = 0..7,
// diagonal rays k = 0..3, orthogonal rays k = 0..3 (functions rather than
// tables, so device code needs no table in global memory).
GZ_HDI int knight_df(int k) { return (int)((0x12211221u >> (4 * k)) & 0xF) * ((k & 4) ? -1 : 1); }
GZ_HDI int knight_dr(int k) { return knight_df((k + 2) & 7); }
GZ_HDI int king_df(int k) { return k == 2 || k == 6 ? 0 : (k == 0 || k == 1 || k == 7) ? 1 : -1; }
GZ_HDI int king_dr(int k) { return king_df((k + 6) & 7); }
GZ_HDI int diag_df(int k) { return k == 0 || k == 3 ? 1 : -1; }
GZ_HDI int diag_dr(int k) { return k < 2 ? 1 : -1; }
GZ_HDI int line_df(int k) { return k == 0 ? 1 : k == 2 ? -1 : 0; }
GZ_HDI int line_dr(int k) { return k == 1 ? 1 : k == 3 ? -1 : 0; }

GZ_HDI bool on_board(int f, int r) { return (unsigned)f < 8u && (unsigned)r < 8u; }

// Is square s attacked by side `by` (+1 / -1)?
GZ_HDI bool attacked(const Pos& p, int s, int by) {
  const int f = file_of(s), r = rank_of(s);
  // pawns of `by` attack diagonally forward (rank + by)
  for (int df = -1; df <= 1; df += 2) {
    const int pf = f + df, pr = r - by;
    if (on_board(pf, pr) && p.sq[pr * 8 + pf] == by * kPawn) return true;
  }
  for (int k = 0; k < 8; ++k) {
    const int nf = f + knight_df(k), nr = r + knight_dr(k);
    if (on_board(nf, nr) && p.sq[nr * 8 + nf] == by * kKnight) return true;
  }
  for (int k = 0; k < 8; ++k) {
    const int nf = f + king_df(k), nr = r + king_dr(k);
    if (on_board(nf, nr) && p.sq[nr * 8 + nf] == by * kKing) return true;
  }
  for (int k = 0; k < 8; ++k) {  // diagonal rays, then orthogonal ones
    const bool diag = k < 4;
    const int df = diag ? diag_df(k) : line_df(k - 4), dr = diag ? diag_dr(k) : line_dr(k - 4);
    const int slider = diag ? kBishop : kRook;
    for (int nf = f + df, nr = r + dr; on_board(nf, nr); nf += df, nr += dr) {
      const int v = p.sq[nr * 8 + nf];
      if (v == 0) continue;
      if (v == by * slider || v == by * kQueen) return true;
      break;
    }
  }
  return false;
}

GZ_HDI int king_square(const Pos& p, int side) {
  for (int s = 0; s < 64; ++s)
    if (p.sq[s] == side * kKing) return s;
  return -1;
}

GZ_HDI void clear_corner_right(Pos& p, int s) {
  if (s == 7) p.castle &= ~0x1u;
  if (s == 0) p.castle &= ~0x2u;
  if (s == 63) p.castle &= ~0x4u;
  if (s == 56) p.castle &= ~0x8u;
}

// Apply a (pseudo-)legal move in place.
GZ_HDI void apply(Pos& p, const Move& m) {
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
  clear_corner_right(p, m.from);
  clear_corner_right(p, m.to);
  p.ep = (type == kPawn && (m.to - m.from == 16 || m.from - m.to == 16)) ? (int8_t)((m.from + m.to) / 2) : (int8_t)-1;
  p.side = (int8_t)-me;
}

// Pseudo-legal moves of the piece of the side to move on square s (none if
// the square holds no such piece), at most `cap` of them: per pawn push,
// double push, captures toward the lower then the higher file, promotions
// Q R B N; knight and king steps k = 0..7, then castling king side, queen
// side; sliders diagonal rays then orthogonal ones.
GZ_HDI int piece_moves(const Pos& p, int s, Move* out, int cap) {
  const int me = p.side;
  int n = 0;
  auto add = [&](int from, int to, int promo) {
    if (n < cap) out[n++] = Move{(int8_t)from, (int8_t)to, (int8_t)promo};
  };
  auto add_pawn = [&](int from, int to) {
    const int last = me > 0 ? 7 : 0;
    if (rank_of(to) == last) {
      add(from, to, kQueen);
      add(from, to, kRook);
      add(from, to, kBishop);
      add(from, to, kKnight);
    } else {
      add(from, to, 0);
    }
  };
  const int v = p.sq[s];
  if (v == 0 || sgn(v) != me) return 0;
  const int type = v * me, f = file_of(s), r = rank_of(s);
  if (type == kPawn) {
    const int r1 = r + me;
    if (!on_board(f, r1)) return 0;
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
    for (int k = 0; k < 8; ++k) {
      const int nf = f + (type == kKnight ? knight_df(k) : king_df(k));
      const int nr = r + (type == kKnight ? knight_dr(k) : king_dr(k));
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
      const int df = k < 4 ? diag_df(k) : line_df(k - 4), dr = k < 4 ? diag_dr(k) : line_dr(k - 4);
      for (int nf = f + df, nr = r + dr; on_board(nf, nr); nf += df, nr += dr) {
        const int tv = p.sq[nr * 8 + nf];
        if (tv != 0 && sgn(tv) == me) break;
        add(s, nr * 8 + nf, 0);
        if (tv != 0) break;
      }
    }
  }
  return n;
}

// Pseudo-legal moves of the side to move, squares ascending, each square's
// in piece_moves' order.  Returns the count; `out` holds 256 and the list
// stops there (reachable chess positions have far fewer; a record with more
// pieces than a game can reach may hit the cap, and it keeps every write in
// bounds).
GZ_HDI int pseudo_moves(const Pos& p, Move* out) {
  int n = 0;
  for (int s = 0; s < 64; ++s) n += piece_moves(p, s, out + n, 256 - n);
  return n;
}

// Does pseudo-legal move m leave the mover's king unattacked?  ks is the
// mover's king square before the move (king_square(p, p.side)); the king
// stands there afterwards unless it is the piece that moves.
GZ_HDI bool move_is_legal(const Pos& p, const Move& m, int ks) {
  Pos q = p;
  apply(q, m);
  const int k = m.from == ks ? m.to : ks;
  return k >= 0 && !attacked(q, k, -p.side);
}

GZ_HDI bool move_is_legal(const Pos& p, const Move& m) { return move_is_legal(p, m, king_square(p, p.side)); }

// Legal moves of the side to move, in pseudo_moves' order; returns the
// count (<= 256).
GZ_HDI int legal_moves(const Pos& p, Move* out) {
  Move ps[256];
  const int np = pseudo_moves(p, ps), ks = king_square(p, p.side);
  int n = 0;
  for (int i = 0; i < np; ++i)
    if (move_is_legal(p, ps[i], ks)) out[n++] = ps[i];
  return n;
}

// Legal moves in place: the first `return` entries of ms are the legal ones
// (ms must hold 256).  One buffer instead of two, for device threads.
GZ_HDI int legal_moves_inplace(const Pos& p, Move* ms) {
  const int np = pseudo_moves(p, ms), ks = king_square(p, p.side);
  int n = 0;
  for (int i = 0; i < np; ++i)
    if (move_is_legal(p, ms[i], ks)) ms[n++] = ms[i];
  return n;
}

// Has the side to move a legal move?  `scratch` holds 256 moves.
GZ_HDI bool has_legal_move(const Pos& p, Move* scratch) {
  Move* ms = scratch;
  const int np = pseudo_moves(p, ms), ks = king_square(p, p.side);
  for (int i = 0; i < np; ++i)
    if (move_is_legal(p, ms[i], ks)) return true;
  return false;
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
GZ_HDI int make_position(uint64_t seed, uint64_t index, int8_t* rec) {
  SplitMix r(mix_seed(seed, 0xC4E55 + index));
  Pos p;
  start_pos(p);
  const int k = (int)r.below(121u);
  Move ms[256];
  for (int ply = 0; ply < k; ++ply) {
    const int n = legal_moves_inplace(p, ms);
    if (n == 0) break;
    Pos q = p;
    apply(q, ms[r.below((uint32_t)n)]);
    if (!has_legal_move(q, ms)) break;
    p = q;
  }
  to_record(p, rec);
  return p.side;
}

// Action index of a move, in the reference's action space of 64 x 73
// (games/chess/chess.cu:94-99, decoded at 127-133): from * 73 + t, where t
// < 64 is the destination square (ordinary moves, castling as the king's
// two-square step, and promotions to a queen) and t >= 64 names an
// underpromotion: 64 + u for a straight pawn push (u = 0 knight, 1 bishop,
// 2 rook, the reference's 64 + piece - KNIGHT), 67 + u for a capture toward
// the lower file, 70 + u toward the higher file.  Every legal move has its
// own index.  (The reference's generator, chess.cu:251-258, marks 64..67 for
// every promoting pawn, queen included, whatever its destination, so it
// cannot tell a capturing promotion from a push.)
GZ_HDI int encode_action(const Move& m) {
  if (m.promo == 0 || m.promo == kQueen) return m.from * 73 + m.to;
  const int dfile = file_of(m.to) - file_of(m.from);
  return m.from * 73 + (dfile == 0 ? 64 : dfile < 0 ? 67 : 70) + (m.promo - kKnight);
}

// The move that action index a names in position p (the inverse of
// encode_action on p's legal moves; no legality check: a must come from
// p's legal list).
GZ_HDI Move decode_action(const Pos& p, int a) {
  const int from = a / 73, t = a % 73;
  Move m;
  m.from = (int8_t)from;
  if (t < 64) {
    m.to = (int8_t)t;
    const bool pawn_to_last = p.sq[from] * p.side == kPawn && rank_of(t) == (p.side > 0 ? 7 : 0);
    m.promo = (int8_t)(pawn_to_last ? kQueen : 0);
  } else {
    const int u = (t - 64) % 3, dir = (t - 64) / 3;  // dir 0 straight, 1 lower file, 2 higher file
    m.to = (int8_t)(from + 8 * p.side + (dir == 0 ? 0 : dir == 1 ? -1 : 1));
    m.promo = (int8_t)(kKnight + u);
  }
  return m;
}

// The legal move with action index a, if any (returns false otherwise).
GZ_HDI bool find_action_with(const Pos& p, int a, Move* out, Move* scratch) {  // scratch holds 256 moves
  if (a < 0 || a >= 64 * 73) return false;
  Move* ms = scratch;
  const int np = pseudo_moves(p, ms);
  for (int i = 0; i < np; ++i)
    if (ms[i].from == a / 73 && encode_action(ms[i]) == a && move_is_legal(p, ms[i])) {
      *out = ms[i];
      return true;
    }
  return false;
}

GZ_HDI bool find_action(const Pos& p, int a, Move* out) {
  Move ms[256];
  return find_action_with(p, a, out, ms);
}

// Game state for the side to move: 0 while it has a legal move; otherwise
// -1 if its king is attacked (checkmate: the side to move has lost) and 2
// for stalemate (a draw).  The 50-move rule, repetitions and insufficient
// material are not tracked.
GZ_HDI int outcome_with(const Pos& p, Move* scratch) {  // scratch holds 256 moves
  if (has_legal_move(p, scratch)) return 0;
  const int k = king_square(p, p.side);
  return k >= 0 && attacked(p, k, -p.side) ? -1 : 2;
}

GZ_HDI int outcome(const Pos& p) {
  Move ms[256];
  return outcome_with(p, ms);
}

}  // namespace chess
}  // namespace gz
