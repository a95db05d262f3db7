// Mapping expressions: parser, position semantics, flattening and walk planning.
// Semantics follow `furiosa-mapping-types/src/dsl.rs:43-277`; the planner is this backend's own.
#include "mapping.hpp"

#include <algorithm>
#include <cctype>
#include <set>
#include <sstream>
#include <unordered_map>

namespace fopt {

int AxisTable::intern(const std::string& n, i64 size) {
  int i = find(n);
  if (i >= 0) {
    if (sizes[i] != size) throw MappingError("axis " + n + " redeclared with a different size");
    return i;
  }
  names.push_back(n);
  sizes.push_back(size);
  return (int)names.size() - 1;
}

// ------------------------------------------------------------------------------------------------
// Parser
// ------------------------------------------------------------------------------------------------
namespace {

struct Tok {
  enum T { Sym, Num, Slash, Pct, Eq, Hash, LP, RP, LB, RB, Comma, End } t;
  std::string s;
  i64 n = 0;
  PadKind pad = PadKind::Top;
};

std::vector<Tok> lex(const std::string& src) {
  std::vector<Tok> out;
  size_t i = 0;
  std::string s = src;
  // Accept an optional `m!` prefix so reference spellings paste verbatim.
  while (i < s.size() && isspace((unsigned char)s[i])) ++i;
  if (s.compare(i, 2, "m!") == 0) i += 2;
  while (i < s.size()) {
    char c = s[i];
    if (isspace((unsigned char)c)) { ++i; continue; }
    if (isalpha((unsigned char)c) || c == '_') {
      size_t j = i;
      while (j < s.size() && (isalnum((unsigned char)s[j]) || s[j] == '_')) ++j;
      out.push_back({Tok::Sym, s.substr(i, j - i)});
      i = j;
      continue;
    }
    if (isdigit((unsigned char)c)) {
      size_t j = i;
      i64 v = 0;
      while (j < s.size() && (isdigit((unsigned char)s[j]) || s[j] == '_')) {
        if (s[j] != '_') v = v * 10 + (s[j] - '0');
        ++j;
      }
      Tok t{Tok::Num, ""};
      t.n = v;
      out.push_back(t);
      i = j;
      continue;
    }
    Tok t{Tok::End, ""};
    switch (c) {
      case '/': t.t = Tok::Slash; break;
      case '%': t.t = Tok::Pct; break;
      case '=': t.t = Tok::Eq; break;
      case '(': t.t = Tok::LP; break;
      case ')': t.t = Tok::RP; break;
      case '[': t.t = Tok::LB; break;
      case ']': t.t = Tok::RB; break;
      case ',': t.t = Tok::Comma; break;
      case '#': {
        t.t = Tok::Hash;
        size_t j = i + 1;
        while (j < s.size() && isspace((unsigned char)s[j])) ++j;
        if (j < s.size() && s[j] == '{') {
          size_t k = s.find('}', j);
          if (k == std::string::npos) throw MappingError("unterminated #{..} in " + src);
          std::string kind = s.substr(j + 1, k - j - 1);
          kind.erase(std::remove_if(kind.begin(), kind.end(), ::isspace), kind.end());
          if (kind == "*") t.pad = PadKind::Top;
          else if (kind == "0") t.pad = PadKind::Zero;
          else if (kind == "!") t.pad = PadKind::Bottom;
          else throw MappingError("unknown padding kind #{" + kind + "}");
          i = k;
        }
        break;
      }
      default:
        throw MappingError(std::string("unexpected character '") + c + "' in mapping " + src);
    }
    out.push_back(t);
    ++i;
  }
  out.push_back({Tok::End, ""});
  return out;
}

NodeP mk(Node::Kind k) {
  auto n = std::make_shared<Node>();
  n->kind = k;
  return n;
}

struct Parser {
  std::vector<Tok> toks;
  size_t p = 0;
  const std::shared_ptr<AxisTable>& axes;
  std::string src;

  const Tok& peek() const { return toks[p]; }
  Tok next() { return toks[p++]; }
  [[noreturn]] void fail(const std::string& why) { throw MappingError(why + " in mapping `" + src + "`"); }

  // Mapping0 := Mapping1 (',' Mapping0)? ','?
  NodeP m0() {
    NodeP left = m1();
    if (peek().t == Tok::Comma) {
      next();
      if (peek().t == Tok::RB || peek().t == Tok::RP || peek().t == Tok::End) return left;
      NodeP right = m0();
      auto n = mk(Node::Pair);
      n->a = left;
      n->b = right;
      n->size = left->size * right->size;
      return n;
    }
    return left;
  }
  i64 num() {
    Tok t = next();
    if (t.t != Tok::Num) fail("expected a number");
    return t.n;
  }
  NodeP m1() {
    NodeP cur = m2();
    for (;;) {
      Tok::T t = peek().t;
      if (t == Tok::Slash) {
        next();
        i64 v = num();
        if (v == 0 || cur->size % v) fail("stride " + std::to_string(v) + " does not divide size " + std::to_string(cur->size));
        auto n = mk(Node::Stride);
        n->a = cur; n->arg = v; n->size = cur->size / v;
        cur = n;
      } else if (t == Tok::Pct) {
        next();
        i64 v = num();
        if (v == 0 || cur->size % v) fail("modulo " + std::to_string(v) + " does not divide size " + std::to_string(cur->size));
        auto n = mk(Node::Modulo);
        n->a = cur; n->arg = v; n->size = v;
        cur = n;
      } else if (t == Tok::Eq) {
        next();
        i64 v = num();
        if (v > cur->size) fail("resize " + std::to_string(v) + " exceeds size " + std::to_string(cur->size));
        auto n = mk(Node::Resize);
        n->a = cur; n->arg = v; n->size = v;
        cur = n;
      } else if (t == Tok::Hash) {
        PadKind k = next().pad;
        i64 v = num();
        if (v < cur->size) fail("padding " + std::to_string(v) + " is below size " + std::to_string(cur->size));
        auto n = mk(Node::Padding);
        n->a = cur; n->arg = v; n->pad = k; n->size = v;
        cur = n;
      } else {
        return cur;
      }
    }
  }
  NodeP m2() {
    Tok t = next();
    if (t.t == Tok::Sym) {
      int a = axes->find(t.s);
      if (a < 0) fail("undeclared axis " + t.s);
      auto n = mk(Node::Symbol);
      n->axis = a; n->arg = axes->sizes[a]; n->size = n->arg;
      return n;
    }
    if (t.t == Tok::Num) {
      auto n = mk(Node::Broadcast);
      n->arg = t.n; n->size = t.n;
      return n;
    }
    if (t.t == Tok::LB || t.t == Tok::LP) {
      NodeP inner = m0();
      Tok c = next();
      if ((t.t == Tok::LB && c.t != Tok::RB) || (t.t == Tok::LP && c.t != Tok::RP)) fail("unbalanced brackets");
      return inner;
    }
    fail("unexpected token");
  }
};

}  // namespace

std::shared_ptr<AxisTable> parse_axes(const std::string& decl) {
  auto t = std::make_shared<AxisTable>();
  std::string s = decl;
  for (auto& c : s)
    if (c == ';') c = ',';
  std::stringstream ss(s);
  std::string item;
  while (std::getline(ss, item, ',')) {
    auto eq = item.find_first_of("=:");
    if (eq == std::string::npos) {
      bool blank = std::all_of(item.begin(), item.end(), ::isspace);
      if (blank) continue;
      throw MappingError("axis declaration `" + item + "` lacks `=`");
    }
    std::string name = item.substr(0, eq), val = item.substr(eq + 1);
    name.erase(std::remove_if(name.begin(), name.end(), ::isspace), name.end());
    val.erase(std::remove_if(val.begin(), val.end(), [](char c) { return isspace((unsigned char)c) || c == '_'; }), val.end());
    if (name.empty() || !isupper((unsigned char)name[0])) throw MappingError("axis name `" + name + "` must start uppercase");
    t->intern(name, std::stoll(val));
  }
  return t;
}

Mapping parse_mapping(const std::string& expr, const std::shared_ptr<AxisTable>& axes) {
  Parser p{lex(expr), 0, axes, expr};
  NodeP root;
  if (p.peek().t == Tok::End) {
    root = mk(Node::Broadcast);
    root->arg = 1;
    root->size = 1;
  } else {
    root = p.m0();
  }
  if (p.peek().t != Tok::End) p.fail("trailing tokens");
  return Mapping{root, axes};
}

// ------------------------------------------------------------------------------------------------
// Printing
// ------------------------------------------------------------------------------------------------
static void print(const Node* n, const AxisTable& ax, std::ostream& o, bool top) {
  switch (n->kind) {
    case Node::Symbol: o << ax.names[n->axis]; break;
    case Node::Broadcast: o << n->arg; break;
    case Node::Stride: print(n->a.get(), ax, o, false); o << " / " << n->arg; break;
    case Node::Modulo: print(n->a.get(), ax, o, false); o << " % " << n->arg; break;
    case Node::Resize: print(n->a.get(), ax, o, false); o << " = " << n->arg; break;
    case Node::Padding:
      print(n->a.get(), ax, o, false);
      o << (n->pad == PadKind::Top ? " # " : n->pad == PadKind::Zero ? " #{0} " : " #{!} ") << n->arg;
      break;
    case Node::Pair:
      o << "[";
      print(n->a.get(), ax, o, false);
      o << ", ";
      print(n->b.get(), ax, o, false);
      o << "]";
      break;
  }
  (void)top;
}

std::string Mapping::to_string() const {
  std::ostringstream o;
  print(root.get(), *axes, o, true);
  return o.str();
}

static void collect_idents(const Node* n, std::vector<int>& out) {
  if (n->kind == Node::Symbol) {
    if (std::find(out.begin(), out.end(), n->axis) == out.end()) out.push_back(n->axis);
    return;
  }
  if (n->a) collect_idents(n->a.get(), out);
  if (n->b) collect_idents(n->b.get(), out);
}

std::vector<int> Mapping::idents() const {
  std::vector<int> v;
  collect_idents(root.get(), v);
  return v;
}

// ------------------------------------------------------------------------------------------------
// Brute-force position semantics (dsl.rs `M::map`)
// ------------------------------------------------------------------------------------------------
static int eval_node(const Node* n, i64 i, std::vector<i64>& c) {
  if (i < 0 || i >= n->size) return -1;
  switch (n->kind) {
    case Node::Symbol: c[n->axis] += i; return 0;
    case Node::Broadcast: return 0;
    case Node::Stride: return eval_node(n->a.get(), i * n->arg, c);
    case Node::Modulo: return eval_node(n->a.get(), i % n->a->size, c);
    case Node::Resize: return eval_node(n->a.get(), i, c);
    case Node::Padding:
      if (i >= n->a->size) return 1 + (int)n->pad;
      return eval_node(n->a.get(), i, c);
    case Node::Pair: {
      int l = eval_node(n->a.get(), i / n->b->size, c);
      if (l != 0) return l;
      return eval_node(n->b.get(), i % n->b->size, c);
    }
  }
  return -1;
}

int Mapping::eval(i64 pos, std::vector<i64>& coord) const {
  coord.assign(axes->names.size(), 0);
  return eval_node(root.get(), pos, coord);
}

// ------------------------------------------------------------------------------------------------
// Flattening into affine factors
// ------------------------------------------------------------------------------------------------
static i64 extent_product(const std::vector<Factor>& g, size_t from) {
  i64 p = 1;
  for (size_t i = from; i < g.size(); ++i) p *= g[i].extent;
  return p;
}

// Position i of the result reads position i*s of g.
static bool apply_stride(std::vector<Factor>& g, i64 s) {
  while (s > 1) {
    if (g.empty()) return false;
    Factor& f = g.back();
    if (s % f.extent == 0) {
      if (f.live < 1) return false;
      s /= f.extent;
      g.pop_back();
    } else if (f.extent % s == 0) {
      if (f.axis >= 0) f.mult *= s;
      f.live = (f.live + s - 1) / s;
      f.extent /= s;
      s = 1;
    } else {
      return false;
    }
  }
  return true;
}

// Keep the first r positions of g.
static bool truncate(std::vector<Factor>& g, i64 r) {
  for (;;) {
    i64 total = extent_product(g, 0);
    if (r == total) return true;
    if (g.empty()) return r == 1;
    i64 w = extent_product(g, 1);
    if (r % w == 0) {
      g[0].extent = r / w;
      g[0].live = std::min(g[0].live, r / w);
      return true;
    }
    if (w % r == 0) {
      if (g[0].live < 1) return false;
      g.erase(g.begin());
      continue;
    }
    return false;
  }
}

static bool pad_to(std::vector<Factor>& g, i64 P, PadKind kind) {
  i64 total = extent_product(g, 0);
  if (P == total) return true;
  if (g.empty()) {
    g.push_back({-1, 0, 1, P, kind});
    return true;
  }
  i64 w = extent_product(g, 1);
  if (P % w) return false;
  g[0].extent = P / w;
  g[0].pad = kind;
  return true;
}

static bool flatten_node(const Node* n, std::vector<Factor>& out) {
  switch (n->kind) {
    case Node::Symbol:
      out = {{n->axis, 1, n->arg, n->arg, PadKind::Top}};
      return true;
    case Node::Broadcast:
      out.clear();
      if (n->arg != 1) out.push_back({-1, 0, n->arg, n->arg, PadKind::Top});
      return true;
    case Node::Pair: {
      std::vector<Factor> l, r;
      if (!flatten_node(n->a.get(), l) || !flatten_node(n->b.get(), r)) return false;
      out = l;
      out.insert(out.end(), r.begin(), r.end());
      return true;
    }
    case Node::Stride:
      return flatten_node(n->a.get(), out) && apply_stride(out, n->arg);
    case Node::Modulo:
    case Node::Resize:
      return flatten_node(n->a.get(), out) && truncate(out, n->arg);
    case Node::Padding:
      return flatten_node(n->a.get(), out) && pad_to(out, n->arg, n->pad);
  }
  return false;
}

bool Mapping::flatten(std::vector<Factor>& out) const {
  out.clear();
  if (!flatten_node(root.get(), out)) return false;
  // Drop single-position factors; they carry neither data nor padding.
  out.erase(std::remove_if(out.begin(), out.end(), [](const Factor& f) { return f.extent == 1; }), out.end());
  return true;
}

// ------------------------------------------------------------------------------------------------
// Atoms: the common refinement of several factor lists. Each axis's coordinate is split at every
// factor boundary (mult, mult*live) seen in any list; when those boundaries form a divisibility
// chain, every factor is a run of whole atoms and every atom's contribution to any memory's offset
// is affine in its digit.
// ------------------------------------------------------------------------------------------------
namespace {

struct Atom {
  int axis;     // -1: broadcast / padding-only digit (never matched across lists)
  i64 base;     // coordinate weight of this atom's digit (axis >= 0)
  i64 radix;    // live digit count
  i64 extent;   // digit range including padding
  long uid;     // identity for axis -1 atoms
};

using AtomKey = std::pair<int, i64>;

struct Refiner {
  std::map<int, std::vector<i64>> bps;
  long next_uid = 1;

  void add(const std::vector<Factor>& fs) {
    for (auto& f : fs)
      if (f.axis >= 0 && f.live > 1) {
        bps[f.axis].push_back(f.mult);
        bps[f.axis].push_back(f.mult * f.live);
      }
  }
  bool finish() {
    for (auto& kv : bps) {
      auto& v = kv.second;
      std::sort(v.begin(), v.end());
      v.erase(std::unique(v.begin(), v.end()), v.end());
      for (size_t i = 1; i < v.size(); ++i)
        if (v[i] % v[i - 1]) return false;
    }
    return true;
  }
  // Atoms of one factor list, outermost first.
  bool refine(const std::vector<Factor>& fs, std::vector<Atom>& out) {
    out.clear();
    for (auto& f : fs) {
      if (f.axis < 0 || f.live <= 1) {
        out.push_back({-1, 0, f.live, f.extent, next_uid++});
        continue;
      }
      auto& v = bps[f.axis];
      auto lo = std::lower_bound(v.begin(), v.end(), f.mult);
      auto hi = std::lower_bound(v.begin(), v.end(), f.mult * f.live);
      if (lo == v.end() || hi == v.end() || *lo != f.mult || *hi != f.mult * f.live) return false;
      std::vector<Atom> inner_first;
      for (auto it = lo; it != hi; ++it) {
        i64 r = *(it + 1) / *it;
        inner_first.push_back({f.axis, *it, r, r, 0});
      }
      // Padding rides on the outermost atom: the factor digit d splits as d = inner + w * outer.
      i64 w = inner_first.back().base / f.mult;
      if (f.extent % w) return false;
      inner_first.back().extent = f.extent / w;
      for (auto it = inner_first.rbegin(); it != inner_first.rend(); ++it) out.push_back(*it);
    }
    return true;
  }
};

// Wire weight of each matched atom of a memory list.
std::map<AtomKey, i64> weights(const std::vector<Atom>& atoms) {
  std::map<AtomKey, i64> w;
  i64 acc = 1;
  for (auto it = atoms.rbegin(); it != atoms.rend(); ++it) {
    if (it->axis >= 0) w[{it->axis, it->base}] = acc;
    acc *= it->extent;
  }
  return w;
}

bool flatten_all(std::initializer_list<const Mapping*> ms, std::vector<std::vector<Factor>>& fs) {
  fs.clear();
  for (auto* m : ms) {
    fs.emplace_back();
    if (!m->flatten(fs.back())) return false;
  }
  return true;
}

}  // namespace

void Walk::coalesce() {
  std::vector<Wheel> w;
  for (auto& x : wheels)
    if (x.extent > 1) w.push_back(x);
  std::vector<Wheel> out;
  for (auto& x : w) {
    if (!out.empty()) {
      Wheel& in = out.back();
      bool ok = in.live == in.extent;
      for (int m = 0; m < nmem && ok; ++m) ok = x.stride[m] == in.stride[m] * in.extent;
      if (ok) {
        in.live = x.live * in.extent;
        in.extent = x.extent * in.extent;
        continue;
      }
    }
    out.push_back(x);
  }
  wheels = out;
}

std::string Walk::to_string() const {
  std::ostringstream o;
  o << "walk{";
  for (auto& w : wheels) {
    o << "(" << w.extent;
    if (w.live != w.extent) o << "/" << w.live;
    for (int m = 0; m < nmem; ++m) o << (m ? "," : ":") << w.stride[m];
    o << ")";
  }
  o << "}";
  return o.str();
}

static Wheel wheel_of(const Atom& a, const std::vector<std::map<AtomKey, i64>>& mems) {
  Wheel w{};
  w.extent = a.extent;
  w.live = a.radix;
  for (size_t m = 0; m < mems.size(); ++m) {
    w.stride[m] = 0;
    if (a.axis >= 0) {
      auto it = mems[m].find({a.axis, a.base});
      if (it != mems[m].end()) w.stride[m] = it->second;
    }
  }
  return w;
}

static std::set<AtomKey> keys_of(const std::vector<Atom>& atoms) {
  std::set<AtomKey> k;
  for (auto& a : atoms)
    if (a.axis >= 0) k.insert({a.axis, a.base});
  return k;
}

bool plan_relayout(const Mapping& src, const Mapping& dst, bool allow_broadcast, Walk& walk) {
  // Structural checks that do not depend on factorisability (op_prep.rs:18-27).
  auto si = src.idents(), di = dst.idents();
  for (int a : si)
    if (std::find(di.begin(), di.end(), a) == di.end())
      throw MappingError("transpose: Src must be covered by the dst stream (axis " + src.axes->names[a] + " missing)");
  if (!allow_broadcast)
    for (int a : di)
      if (std::find(si.begin(), si.end(), a) == si.end())
        throw MappingError("transpose: Dst adds axis " + dst.axes->names[a] + " but broadcast is not allowed");

  std::vector<std::vector<Factor>> fs;
  if (!flatten_all({&src, &dst}, fs)) return false;
  Refiner R;
  R.add(fs[0]);
  R.add(fs[1]);
  if (!R.finish()) return false;
  std::vector<Atom> sa, da;
  if (!R.refine(fs[0], sa) || !R.refine(fs[1], da)) return false;
  auto dk = keys_of(da);
  for (auto& a : sa)
    if (a.axis >= 0 && a.radix > 1 && !dk.count({a.axis, a.base})) return false;  // src bits dst lacks
  std::vector<std::map<AtomKey, i64>> mems{weights(sa)};
  walk.nmem = 1;
  walk.wheels.clear();
  for (auto it = da.rbegin(); it != da.rend(); ++it) walk.wheels.push_back(wheel_of(*it, mems));
  walk.coalesce();
  return (int)walk.wheels.size() <= kMaxWheels;
}

std::vector<i64> relayout_table(const Mapping& src, const Mapping& dst, bool allow_broadcast) {
  auto si = src.idents();
  std::map<std::vector<i64>, i64> where;
  std::vector<i64> c;
  for (i64 p = 0; p < src.size(); ++p) {
    if (src.eval(p, c) != 0) continue;
    std::vector<i64> key;
    for (int a : si) key.push_back(c[a]);
    where.emplace(key, p);  // first (lowest) wire position wins for a broadcast src
  }
  std::vector<i64> t(dst.size(), -1);
  for (i64 q = 0; q < dst.size(); ++q) {
    if (dst.eval(q, c) != 0) continue;
    std::vector<i64> key;
    for (int a : si) key.push_back(c[a]);
    auto it = where.find(key);
    if (it == where.end()) {
      if (!allow_broadcast) throw MappingError("transpose: dst cell has no source element");
      continue;
    }
    t[q] = it->second;
  }
  return t;
}

bool plan_reduce(const Mapping& src, const Mapping& dst, bool allow_broadcast, FoldPlan& plan) {
  auto si = src.idents(), di = dst.idents();
  for (int a : di)
    if (std::find(si.begin(), si.end(), a) == si.end() && !allow_broadcast)
      throw MappingError("reduce: Dst adds axes absent from the source; pass allow_broadcast=true for reduce-then-broadcast");
  std::vector<std::vector<Factor>> fs;
  if (!flatten_all({&src, &dst}, fs)) return false;
  Refiner R;
  R.add(fs[0]);
  R.add(fs[1]);
  if (!R.finish()) return false;
  std::vector<Atom> sa, da;
  if (!R.refine(fs[0], sa) || !R.refine(fs[1], da)) return false;
  std::vector<std::map<AtomKey, i64>> mems{weights(sa)};
  auto dk = keys_of(da);
  plan.nmem = 1;
  plan.out.nmem = plan.residue.nmem = 1;
  plan.out.wheels.clear();
  plan.residue.wheels.clear();
  for (auto it = da.rbegin(); it != da.rend(); ++it) plan.out.wheels.push_back(wheel_of(*it, mems));
  for (auto it = sa.rbegin(); it != sa.rend(); ++it) {
    if (it->axis >= 0 && dk.count({it->axis, it->base})) continue;
    // A residue atom: axis atoms dst drops, and src broadcast digits (they fold duplicates, as the
    // reference's live-residue walk does).
    Wheel w{};
    w.extent = it->extent;
    w.live = it->radix;
    if (it->axis >= 0) {
      w.stride[0] = mems[0].at({it->axis, it->base});
    } else {
      // axis -1 atoms are unmatched; recover the weight by position.
      i64 acc = 1;
      for (auto jt = sa.rbegin(); jt != it; ++jt) acc *= jt->extent;
      w.stride[0] = acc;
    }
    plan.residue.wheels.push_back(w);
  }
  plan.out.coalesce();
  plan.residue.coalesce();
  if (plan.residue.live_positions() == 0) throw MappingError("reduce/contraction: residue must have a live cell to fold");
  return (int)plan.out.wheels.size() <= kMaxWheels && (int)plan.residue.wheels.size() <= kMaxWheels;
}

bool plan_contraction(const Mapping& lhs, const Mapping& rhs, const Mapping& pre_reduce, const Mapping& out,
                      FoldPlan& plan, const Mapping* extra) {
  std::vector<std::vector<Factor>> fs;
  if (!flatten_all({&lhs, &rhs, &pre_reduce, &out, extra ? extra : &out}, fs)) return false;
  Refiner R;
  for (auto& f : fs) R.add(f);
  if (!R.finish()) return false;
  std::vector<Atom> la, ra, pa, oa, xa;
  if (!R.refine(fs[0], la) || !R.refine(fs[1], ra) || !R.refine(fs[2], pa) || !R.refine(fs[3], oa) ||
      !R.refine(fs[4], xa))
    return false;
  std::vector<std::map<AtomKey, i64>> mems{weights(la), weights(ra)};
  if (extra) mems.push_back(weights(xa));
  auto ok = keys_of(oa);
  plan.nmem = (int)mems.size();
  plan.out.nmem = plan.residue.nmem = plan.nmem;
  plan.out.wheels.clear();
  plan.residue.wheels.clear();
  for (auto it = oa.rbegin(); it != oa.rend(); ++it) plan.out.wheels.push_back(wheel_of(*it, mems));
  for (auto it = pa.rbegin(); it != pa.rend(); ++it) {
    if (it->axis >= 0 && ok.count({it->axis, it->base})) continue;
    if (it->axis < 0 && it->radix <= 1) {
      // a padding-only digit of pre_reduce: only digit 0 is live
      Wheel w{};
      w.extent = it->extent;
      w.live = 1;
      plan.residue.wheels.push_back(w);
      continue;
    }
    plan.residue.wheels.push_back(wheel_of(*it, mems));
  }
  // Every live operand atom must be either an output or a contracted coordinate.
  auto pk = keys_of(pa);
  for (auto* v : {&la, &ra})
    for (auto& a : *v)
      if (a.axis >= 0 && a.radix > 1 && !pk.count({a.axis, a.base}) && !ok.count({a.axis, a.base}))
        throw MappingError("contraction: operand axis absent from both the union and the output");
  plan.out.coalesce();
  plan.residue.coalesce();
  if (plan.residue.live_positions() == 0) throw MappingError("reduce/contraction: residue must have a live cell to fold");
  return (int)plan.out.wheels.size() <= kMaxWheels && (int)plan.residue.wheels.size() <= kMaxWheels;
}

i64 window_base(const Mapping& base, const std::vector<std::string>& axis_names, const std::vector<i64>& coords) {
  if (axis_names.empty()) return 0;
  std::vector<i64> want(base.axes->names.size(), 0);
  for (size_t i = 0; i < axis_names.size(); ++i) {
    int a = base.axes->find(axis_names[i]);
    if (a < 0) throw MappingError("window offset names unknown axis " + axis_names[i]);
    want[a] = coords[i];
  }
  std::vector<Factor> fs;
  std::vector<i64> c;
  if (base.flatten(fs)) {
    i64 pos = 0, w = 1;
    for (auto it = fs.rbegin(); it != fs.rend(); ++it) {
      i64 d = it->axis >= 0 ? (want[it->axis] / it->mult) % it->live : 0;
      pos += d * w;
      w *= it->extent;
    }
    if (base.eval(pos, c) == 0 && c == want) return pos;
  }
  for (i64 p = 0; p < base.size(); ++p)
    if (base.eval(p, c) == 0 && c == want) return p;
  throw MappingError("transpose: partial-view offset must land on a live cell of its base mapping");
}

RankWalk rank_walk(const Mapping& m) {
  std::vector<Factor> fs;
  if (!m.flatten(fs)) throw MappingError("transmute: mapping " + m.to_string() + " is not affine-factorisable");
  RankWalk r;
  for (auto it = fs.rbegin(); it != fs.rend(); ++it) {
    r.extent.push_back(it->extent);
    r.live.push_back(it->live);
  }
  return r;
}

}  // namespace fopt
