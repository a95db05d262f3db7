// Mapping expressions and walk plans for the B200 backend (host side).
//
// A mapping expression (the `m![...]` language of furiosa-mapping) says where every logical element
// of a tensor sits in its packed device image. This file restates the open position semantics of
// `furiosa-mapping-types/src/dsl.rs:43-277` (Symbol / Stride / Modulo / Resize / Padding / Pair /
// Broadcast `map`) and derives, from two or more mappings, the odometer walks the CUDA kernels run.
// The walk derivation is our own factoriser: the reference's `sequence()` lives in a closed prebuilt
// library (`furiosa-mapping/src/lib.rs:107-116`), so only its observable result -- "the value at a
// logical index is preserved" (`storage/buf.rs:257-313`) -- is reproduced, not its algorithm.
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace fopt {

using i64 = int64_t;

// `furiosa-mapping-types/src/lib.rs:563-573`: Bottom < Zero < Top.
enum class PadKind : int { Bottom = 0, Zero = 1, Top = 2 };

struct MappingError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

// One node of the expression tree (`furiosa-mapping-types/src/lib.rs:144-195`).
struct Node {
  enum Kind { Symbol, Stride, Modulo, Resize, Padding, Pair, Broadcast } kind;
  int axis = -1;       // Symbol: index into the axis table
  i64 arg = 0;         // Symbol: declared size; Stride/Modulo/Resize/Padding: the operand; Broadcast: size
  PadKind pad = PadKind::Top;
  std::shared_ptr<Node> a, b;  // inner (a) or pair (a = left/major, b = right/minor)
  i64 size = 0;                // cached cell count (`Mapping::size`, lib.rs:222-232)
};
using NodeP = std::shared_ptr<Node>;

// Axis names and declared sizes, shared by every mapping parsed against the same table.
struct AxisTable {
  std::vector<std::string> names;
  std::vector<i64> sizes;
  int find(const std::string& n) const {
    for (size_t i = 0; i < names.size(); ++i)
      if (names[i] == n) return (int)i;
    return -1;
  }
  int intern(const std::string& n, i64 size);
};

// A flattened factor of a mapping: one mixed-radix digit of the wire position. Digit `d` in
// `[0, extent)` is live when `d < live` and then contributes `d * mult` to the coordinate of `axis`
// (`axis == -1`: a broadcast digit that contributes nothing).
struct Factor {
  int axis;
  i64 mult;
  i64 live;
  i64 extent;
  PadKind pad;
};

struct Mapping {
  NodeP root;
  std::shared_ptr<AxisTable> axes;
  i64 size() const { return root->size; }
  std::string to_string() const;
  // Flattens into factors, outermost first; returns false when some node is not a product of
  // affine digits (a "composite" in the reference's vocabulary).
  bool flatten(std::vector<Factor>& out) const;
  // Brute-force `M::map(i)` (dsl.rs): fills `coord` (one entry per axis of the table, summed
  // contributions) and returns 0 for a live cell, 1 + PadKind for padding, -1 out of bounds.
  int eval(i64 pos, std::vector<i64>& coord) const;
  // Distinct axes referenced (`Mapping::idents`, lib.rs:359-382), first-encounter order.
  std::vector<int> idents() const;
};

// Parses the `m!` grammar (`furiosa-mapping-macro/src/parser/parser.lalrpop`): comma pairs are
// right-associative, postfix `/ n`, `% n`, `= n`, `# n`, `#{*} n`, `#{0} n`, `#{!} n` bind left to
// right, `[..]` / `(..)` group, a bare number is a broadcast. `axes` declares sizes: "A=8, B=512".
Mapping parse_mapping(const std::string& expr, const std::shared_ptr<AxisTable>& axes);
std::shared_ptr<AxisTable> parse_axes(const std::string& decl);

// ---------------------------------------------------------------------------------------------
// Walks. A walk enumerates the positions of a stream mapping as an odometer over wheels
// (innermost first). Wheel `w` has digit range `[0, extent)`, is live while the digit is `< live`,
// and moves each memory's offset by `stride[m]` per step.
// ---------------------------------------------------------------------------------------------
constexpr int kMaxWheels = 16;
constexpr int kMaxMems = 3;

struct Wheel {
  i64 extent;
  i64 live;
  i64 stride[kMaxMems];
};

struct Walk {
  std::vector<Wheel> wheels;  // innermost first
  int nmem = 1;
  i64 positions() const {
    i64 p = 1;
    for (auto& w : wheels) p *= w.extent;
    return p;
  }
  i64 live_positions() const {
    i64 p = 1;
    for (auto& w : wheels) p *= w.live;
    return p;
  }
  // Merges adjacent wheels whose strides continue each other and drops extent-1 wheels.
  void coalesce();
  std::string to_string() const;
};

// Relayout (`BufStorage::transpose`, buf.rs:257-313): walk over the dst positions; memory 0 = src.
// Throws MappingError if Src is not covered by Dst, or Dst adds live axes and !allow_broadcast.
// Returns false (walk left empty) when the mappings are not affine-factorisable; the caller then
// builds an explicit offset table with `relayout_table`.
bool plan_relayout(const Mapping& src, const Mapping& dst, bool allow_broadcast, Walk& walk);
// Explicit per-dst-position src offset (-1 for dead positions) by brute-force index matching.
std::vector<i64> relayout_table(const Mapping& src, const Mapping& dst, bool allow_broadcast);

// Per-output-cell fold plan (`ReadPlan`, buf.rs:680-753) for reduce and contraction.
//   out:     walk over the output positions (dead = padding cell, keeps identity / zero);
//   residue: walk over the folded (reduced / contracted) coordinates in the reference's residue
//            order (ascending wire order of the residue mapping), live digits only fold.
// Memory m of each walk is operand m.
struct FoldPlan {
  Walk out;
  Walk residue;
  int nmem = 1;
};
// reduce (buf.rs:331-376): src -> dst; dst axes absent in src broadcast (needs allow_broadcast).
bool plan_reduce(const Mapping& src, const Mapping& dst, bool allow_broadcast, FoldPlan& plan);
// contraction (buf.rs:401-447): operands lhs, rhs; contracted = pre_reduce minus out.
// `extra` (optional) adds memory 2 to the output walk: e.g. a per-channel scale vector `[N]`.
bool plan_contraction(const Mapping& lhs, const Mapping& rhs, const Mapping& pre_reduce,
                      const Mapping& out, FoldPlan& plan, const Mapping* extra = nullptr);

// `window_base` (buf.rs:760-781): wire position of the logical offset `coord` (one entry per axis
// name listed in `axis_names`) in `base`.
i64 window_base(const Mapping& base, const std::vector<std::string>& axis_names,
                const std::vector<i64>& coords);

// Live-rank walk for `transmute` (buf.rs:592-613, 785-795): the k-th live element of src (wire
// order) lands on the k-th live position of dst.
struct RankWalk {
  std::vector<i64> extent, live;  // innermost first
};
RankWalk rank_walk(const Mapping& m);

}  // namespace fopt
