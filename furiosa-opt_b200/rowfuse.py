"""Row programs: engine-chain fusion across a row reduction.

The reference runs a normalisation or a per-token quantisation as a chain of storage ops, each a
full pass over memory: a map, a row `reduce` (`BufStorage::reduce`, furiosa-opt-std/src/storage/
buf.rs:331-376), a map of the per-row result, a broadcast `transpose` of it back over the rows
(buf.rs:257-313) and a zip with the original values (buf.rs:203-250). Deferred elementwise values,
lazy broadcasts and lazy row reductions keep that chain as a graph; when a value at the end of it
is needed, `try_row_program` lowers the graph to one `fopt_row_plan` and the library runs it as one
kernel with a CTA per row: the row is read once, every reduction of it is folded in turn, the
per-row scalars between them are computed, and the final program writes the row.

Graph nodes are storages:
  * element nodes (one value per element of a [rows, W] row-major tensor): materialised storages
    (leaves), lazy broadcasts of per-row scalars (slots), lazy broadcasts of anything else (leaves
    read through the broadcast index), and deferred elementwise values (expressions over their
    origin inputs);
  * scalar nodes (one value per row): lazy row reductions (FOLD slots over an element node),
    deferred elementwise values over scalar nodes (SCALAR slots) and materialised [rows] storages
    (LOAD slots).
Every FOLD slot is one pass over the row; the final program is the last pass. Element
sub-expressions that depend on no slot and that a later pass needs are computed in the first pass
and held in registers (the SwiGLU activation between its absolute-max pass and its quantisation
pass, for example), instead of re-reading and recomputing them.
"""
from __future__ import annotations

import ctypes as C

from . import _lib, ops
from ._lib import check


class _NoRow(Exception):
    pass


_PROGS = {}  # element-program signature -> composed program


def _is_lazy(s, kind):
    return s.lazy is not None and s.lazy[0] == kind


def _children(s):
    """(program, inputs) of a deferred elementwise storage: its origin, else its flat form."""
    _, prog, leaves, origin = s.lazy
    return origin if origin is not None else (prog, leaves)


class _Planner:
    def __init__(self, be, rows: int, W: int):
        self.be, self.rows, self.W = be, rows, W
        self.leaves = []        # (Storage whose memory is read, dtype, bcast code)
        self.leaf_of = {}       # id(element node) -> leaf index
        self.slots = []         # dicts: kind, node, ...
        self.slot_of = {}       # id(scalar node) -> slot index
        self.leaf_only = {}     # id(element node) -> True when no slot feeds it
        self.keep = []          # storages referenced by the plan (kept alive until the launch)

    # ---- discovery ----
    def elem(self, x) -> bool:
        """Registers element node x; returns whether it depends on no slot."""
        key = id(x)
        if key in self.leaf_only:
            return self.leaf_only[key]
        self.keep.append(x)
        n = self.rows * self.W
        if x.n != n:
            raise _NoRow
        if x.lazy is None:
            self._leaf(x, x, 0)
            only = True
        elif x.lazy[0] == "bcast":
            src, code = x.lazy[1], x.lazy[4]
            if code == self.W and src.n == self.rows:
                self.scalar(src)
                only = False
            else:
                self.be._force(src)  # a broadcast of a value written out: read it through the index
                self._leaf(x, src, code)
                only = True
        elif x.lazy[0] == "ew":
            _, inputs = _children(x)
            only = all([self.elem(c) for c in inputs])
        else:
            raise _NoRow
        self.leaf_only[key] = only
        return only

    def _leaf(self, node, mem, code):
        if id(node) not in self.leaf_of:
            if len(self.leaves) >= _lib.ROW_MAX_LEAVES:
                raise _NoRow
            self.leaf_of[id(node)] = len(self.leaves)
            self.leaves.append((mem, mem.dtype, code))

    def scalar(self, s) -> int:
        key = id(s)
        if key in self.slot_of:
            return self.slot_of[key]
        self.keep.append(s)
        if s.n != self.rows:
            raise _NoRow
        if s.lazy is None:
            slot = dict(kind=_lib.ROW_LOAD, node=s)
        elif s.lazy[0] == "red":
            _, src, op, bits, _, _, rows, W = s.lazy
            if rows != self.rows or W != self.W or s.dtype not in ("f32", "i32"):
                raise _NoRow
            self.elem(src)
            slot = dict(kind=_lib.ROW_FOLD, node=s, src=src, op=op, bits=bits)
        elif s.lazy[0] == "ew":
            if s.dtype not in ("f32", "i32"):
                raise _NoRow
            _, inputs = _children(s)
            for c in inputs:
                self.scalar(c)
            slot = dict(kind=_lib.ROW_SCALAR, node=s)
        else:
            raise _NoRow
        if len(self.slots) >= _lib.ROW_MAX_SLOTS:
            raise _NoRow
        self.slot_of[key] = len(self.slots)
        self.slots.append(slot)
        return self.slot_of[key]

    # ---- held values ----
    def frontier(self, root_inputs, out: list, seen: set):
        """Slot-free expression nodes a pass over these inputs reads (it stops at them)."""
        for x in root_inputs:
            if id(x) in seen:
                continue
            seen.add(id(x))
            if id(x) in self.leaf_of or not _is_lazy(x, "ew"):
                continue
            if self.leaf_only[id(x)]:
                out.append(x)
            else:
                self.frontier(_children(x)[1], out, seen)

    # ---- programs ----
    def elem_prog(self, root_prog, root_inputs, n_in, reg_of):
        """Composes the element program of a pass (or of a held value) over n_in input registers;
        reg_of(node) returns the register of a node that is an input, or None to expand it.
        Memoised on the tree the program computes (programs and input registers): two graphs with
        the same tree compute the same function of the same registers."""
        sigs = {}

        def sig(x):
            if id(x) not in sigs:
                r = reg_of(x)
                if r is not None:
                    sigs[id(x)] = r
                else:
                    prog, inputs = _children(x)
                    sigs[id(x)] = (bytes(prog), tuple(sig(c) for c in inputs))
            return sigs[id(x)]

        key = (n_in, bytes(root_prog), tuple(sig(c) for c in root_inputs))
        if key in _PROGS:
            return _PROGS[key]
        built = self._elem_prog(root_prog, root_inputs, n_in, reg_of)
        if len(_PROGS) >= 4096:
            _PROGS.clear()
        _PROGS[key] = built
        return built

    def _elem_prog(self, root_prog, root_inputs, n_in, reg_of):
        b = ops.Prog(n_in)
        memo = {}

        def reg(x):
            if id(x) in memo:
                return memo[id(x)]
            r = reg_of(x)
            if r is None:
                prog, inputs = _children(x)
                r = ops.inline(b, prog, [reg(c) for c in inputs])
            memo[id(x)] = r
            return r

        return b.build(ops.inline(b, root_prog, [reg(c) for c in root_inputs]))


def _cheap(pl, x) -> bool:
    leaves = set()

    def walk(n, depth):
        if id(n) in pl.leaf_of:
            leaves.add(id(n))
            return 0
        prog, inputs = _children(n)
        return prog.n_insn + sum(walk(c, depth + 1) for c in inputs)

    insns = walk(x, 0)
    return insns <= 2 and len(leaves) == 1


class RowBuild:
    """A lowered row program: the ctypes plan (slot outputs not yet set), the scalar storages its
    FOLD / SCALAR slots compute (in slot order, None for LOAD slots) and what keeps it alive."""

    def __init__(self, plan, slot_nodes, keep):
        self.plan, self.slot_nodes, self.keep = plan, slot_nodes, keep


def build_row_program(be, prog, leaves, out, origin):
    """Lowers the elementwise value `out` = prog(leaves) to a row plan when one of its leaves is a
    per-row broadcast of a value still to be computed from a row reduction; None otherwise."""
    W = None
    for leaf in leaves:
        if _is_lazy(leaf, "bcast") and leaf.lazy[4] > 0 and leaf.lazy[1].lazy is not None \
                and leaf.lazy[1].lazy[0] in ("ew", "red"):
            W = leaf.lazy[4]
            break
    if W is None or out.n % W or W % 8 or W > 32768:
        return None
    rows = out.n // W
    root_prog, root_inputs = origin if origin is not None else (prog, leaves)
    pl = _Planner(be, rows, W)
    try:
        for x in root_inputs:
            pl.elem(x)
        if not any(s["kind"] == _lib.ROW_FOLD for s in pl.slots):
            return None
        # passes: every FOLD slot in slot order, then the final program
        passes = [[s["src"]] for s in pl.slots if s["kind"] == _lib.ROW_FOLD] + [root_inputs]
        held, seen = [], set()
        for inputs in passes[1:]:
            pl.frontier(inputs, held, seen)
        # a value a couple of instructions from one leaf (a cast) is cheaper to recompute from the
        # leaf kept raw, which takes fewer registers than the 32-bit value
        held = [x for x in held if not _cheap(pl, x)]
        KC = (W + 2047) // 2048
        if len(held) > _lib.ROW_MAX_HELD or len(held) * 8 * KC > 64:
            held = []
        nL, nH, nS = len(pl.leaves), len(held), len(pl.slots)
        if nL + nH + nS > 16:
            return None
        held_idx = {id(h): i for i, h in enumerate(held)}

        def elem_reg(x):
            if id(x) in pl.leaf_of:
                return pl.leaf_of[id(x)]
            if id(x) in held_idx:
                return nL + held_idx[id(x)]
            if _is_lazy(x, "bcast"):  # a per-row scalar
                return nL + nH + pl.slot_of[id(x.lazy[1])]
            return None

        def leaf_reg(x):
            return pl.leaf_of.get(id(x))

        ident = ops.Prog(1).build(0)  # returns its input
        keep = list(pl.keep)

        def kept(p):
            keep.append(p)
            return C.pointer(p)

        plan = _lib.RowPlan()
        plan.n_leaves, plan.n_held, plan.n_slots = nL, nH, nS
        for k, (mem, dt, code) in enumerate(pl.leaves):
            plan.leaf[k] = mem.addr
            plan.leaf_dtype[k] = _lib.DTYPES[dt]
            plan.leaf_bcast[k] = code
        for h, x in enumerate(held):
            plan.held[h] = kept(pl.elem_prog(ident, [x], nL, leaf_reg))
        slot_nodes = []
        for j, sl in enumerate(pl.slots):
            slot, node = plan.slot[j], sl["node"]
            slot.kind = sl["kind"]
            slot.dtype = _lib.DTYPES[node.dtype]
            if sl["kind"] == _lib.ROW_LOAD:
                slot.src = node.addr
                slot_nodes.append(None)
                continue
            if sl["kind"] == _lib.ROW_FOLD:
                slot.op = _lib.REDUCE_OPS[sl["op"]]
                slot.identity_bits = sl["bits"]
                slot.prog = kept(pl.elem_prog(ident, [sl["src"]], nL + nH + nS, elem_reg))
            else:
                sprog, sinputs = _children(node)
                b = ops.Prog(j)
                slot.prog = kept(b.build(ops.inline(b, sprog, [pl.slot_of[id(c)] for c in sinputs])))
            slot_nodes.append(node)
        plan.final_prog = kept(pl.elem_prog(root_prog, root_inputs, nL + nH + nS, elem_reg))
    except (_NoRow, ValueError):
        return None
    plan.out_dtype = _lib.DTYPES[out.dtype]
    plan.rows, plan.row_len = rows, W
    return RowBuild(plan, slot_nodes, keep)


def try_row_program(be, prog, leaves, out, origin) -> bool:
    """Runs `out` = prog(leaves) as a row program (see `build_row_program`); False when that does
    not apply (nothing has run then). The per-row scalars it computes are written out and stop
    being lazy."""
    rb = build_row_program(be, prog, leaves, out, origin)
    if rb is None:
        return False
    plan = rb.plan
    outs = []
    for j, node in enumerate(rb.slot_nodes):
        if node is None:
            continue
        p = C.c_void_p()
        check(_lib.lib().fopt_alloc_uninit(be.ctx, node.nbytes, C.byref(p)), be.ctx)
        outs.append((node, p))
        plan.slot[j].out = p
    plan.out = out._ptr
    st = _lib.lib().fopt_row_program(be.ctx, C.byref(plan))
    if st != 0:
        for _, p in outs:
            _lib.lib().fopt_free(be.ctx, p)
        if st == _lib.FOPT_ERR_UNSUPPORTED:
            return False
        check(st, be.ctx)
    for node, p in outs:  # the per-row scalars now hold their values
        node.lazy = None
        node._ptr = p
        node._capture = be._capturing  # as `Storage._alloc` records it
    return True
