"""Single-token (decode) fusion patterns of the ``cuda-b200`` planner.

Each pattern recognises a structure that ``LlamaDecoderStep`` builds
(chomikgrad/llama.py:457-543) -- checking operators, operand identity,
constant values, consumers and runtime dtypes -- and replaces it with one or
two fused kernels.  Anything that does not match exactly stays on the
generic path, so the fusions never change what a graph computes.

Patterns (anchor node in brackets):

* attention block [sdpa]: rms_norm -> q/k/v linears (one GEMV over the three
  weights) -> RoPE(q, k) at ``position`` -> write-mask cache blend
  ``cache*(1-wm) + key*wm`` (:511-512) -> masked softmax attention (:514-525)
  => ``cb_gemv`` + ``cb_decode_attention`` (cache updated in place when the
  cache is a dynamic input used only by the blend);
* SwiGLU [mul]: ``silu(x @ Wg^T) * (x @ Wu^T)`` (:289-291, :371-380)
  => ``cb_gemv`` with the SILU_MUL epilogue;
* residual linear [add]: ``h + x @ W^T`` (:529-535) => ``cb_gemv`` RESIDUAL;
* plain linear [matmul]: ``x @ W^T`` => ``cb_gemv`` STORE (+ argmax when it
  is a 2-D program output -- the logits, :537-541).

Linear inputs that are ``rms_norm`` lowerings are normalised inside the GEMV
prologue; ``rms_norm(gather(table, ids))`` (layer 0) reads a per-row table of
the norm's sqrt term computed once per program, so decode never repeats the
reference's sequential bfloat16 sum.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

from . import _lib
from .planner import F32, View, contiguous_strides, is_ew, kind

PREFETCH_CAP = 48 << 20        # bytes of one weight step prefetched ahead
PREFETCH_OUTSTANDING = 96 << 20  # bytes prefetched but not yet consumed


@dataclass
class Linear:
    node: object          # MATMUL node
    weight: object        # 2-D weight leaf (HF (out, in) layout)
    x: object             # the matmul's left operand
    source: object        # x with views stripped
    k: int
    n: int


def _strip_views(node, size: int):
    """Follow reshape/permute nodes that keep a single-token vector contiguous."""
    while kind(node) in ("reshape", "permute"):
        if kind(node) == "permute":
            parent = node.inputs[0]
            kept = [a for a in node.arg if parent.shape[a] != 1]
            if kept != sorted(kept):
                break
        node = node.inputs[0]
    return node if int(np.prod(node.shape)) == size else None


class DecodeFusion:
    def __init__(self, planner) -> None:
        self.p = planner
        self.units: Dict[object, object] = {}
        self.table_reads = set()   # consumers that read a gather through its table
        self._norm_tables: Dict[object, object] = {}

    # ---------------------------------------------------------------- util
    def uses(self, node) -> List[object]:
        return self.p.consumers.get(node, [])

    def only_used_by(self, node, *users) -> bool:
        mine = self.uses(node)
        return (node not in self.p.output_set and len(mine) == len(users)
                and all(any(m is u for u in users) for m in mine))

    def is_one(self, node) -> bool:
        value = self.p._const(node)
        return value is not None and value == 1.0

    def linear(self, node) -> Optional[Linear]:
        if kind(node) != "matmul":
            return None
        x, t = node.inputs
        if kind(t) != "permute" or tuple(t.arg) != (1, 0):
            return None
        w = t.inputs[0]
        if w.op is not None or len(w.shape) != 2 or w in self.p.dynamic or not w.cache_native:
            return None
        if self.p.rdt(w).name not in ("bfloat16", "float32"):
            return None
        n_out, k = w.shape
        if int(np.prod(x.shape[:-1])) != 1 or x.shape[-1] != k:
            return None
        if self.p.rdt(node) != F32 or self.p.rdt(x).name not in ("bfloat16", "float32"):
            return None
        source = _strip_views(x, k)
        if source is None:
            return None
        return Linear(node, w, x, source, k, n_out)

    # ---------------------------------------------------------------- apply
    def apply(self) -> None:
        p = self.p
        linears = {n: l for n in p.order if (l := self.linear(n)) is not None}
        self.linears = linears
        done = set()
        for node in p.order:
            if node in p._low and p._low[node][0] == "sdpa":
                unit = self.attention_block(node)
                if unit is not None:
                    done.update(unit)
        for node in p.order:
            if is_ew(node, "mul") and node not in p.claimed:
                unit = self.swiglu(node)
                if unit is not None:
                    done.update(unit)
        for node in p.order:
            if is_ew(node, "add") and node not in p.claimed:
                self.residual(node, done)
        for node, lin in linears.items():
            if node not in done and node not in p.claimed:
                self.plain(lin)
        # a gather read only through table lookups is never materialised
        for node in p.order:
            if self.gathered_table(node) is not None and node not in p.output_set:
                if self.uses(node) and all(u in self.table_reads for u in self.uses(node)):
                    p.claimed.add(node)
        p.units = self.units

    # ------------------------------------------------------- x / norm input
    def input_spec(self, lins: Sequence[Linear]):
        """How the GEMV reads x: ('value', view) | ('norm', ...) resolved at emit time."""
        src = lins[0].source
        if any(l.source is not src for l in lins):
            return None
        low = self.p._low.get(src)
        if low is not None and low[0] == "rms_norm":
            users = self.uses(src)
            # the norm output may be consumed through views only by these linears
            reach = set()
            stack = list(users)
            while stack:
                u = stack.pop()
                if kind(u) in ("reshape", "permute") and u not in self.p.output_set:
                    stack.extend(self.uses(u))
                else:
                    reach.add(u)
            if src not in self.p.output_set and reach == {l.node for l in lins}:
                if self.gathered_table(low[1][0]) is not None:
                    self.table_reads.add(src)
                return ("norm", src)
        return ("value", lins[0].x)

    def claim_views(self, lins: Sequence[Linear], spec) -> None:
        if spec[0] != "norm":
            return
        stack = [spec[1]]
        while stack:
            n = stack.pop()
            self.p.claimed.add(n)
            stack.extend(u for u in self.uses(n) if kind(u) in ("reshape", "permute"))

    def gemv_args(self, lins: Sequence[Linear], spec, epilogue: int):
        """Common cb_gemv arguments; views resolved lazily in emit()."""
        return dict(lins=lins, spec=spec, epilogue=epilogue)

    # ---------------------------------------------------------- attention
    def _blend(self, node, cache_shape):
        """(cache_leaf, new_row, wm, one_minus_node, nodes) for cache*(1-wm) + row*wm."""
        if not is_ew(node, "add"):
            return None
        left, right = node.inputs
        if not (is_ew(left, "mul") and is_ew(right, "mul")):
            return None
        cache, keep = left.inputs
        row, wm = right.inputs
        if not is_ew(keep, "sub") or not self.is_one(keep.inputs[0]) or keep.inputs[1] is not wm:
            return None
        if cache.op is not None or tuple(cache.shape) != cache_shape:
            return None
        kv = self.p.kv_dtypes()
        if self.p.rdt(cache) not in kv or self.p.rdt(left) not in kv or any(
                self.p.rdt(n) != F32 for n in (right, node)):
            return None
        ctx = cache_shape[2]
        if tuple(wm.shape) != (1, 1, ctx, 1) or self.p.rdt(wm).name not in ("float32", "bfloat16", "float16"):
            return None
        if not (self.only_used_by(left, node) and self.only_used_by(right, node)
                and self.only_used_by(keep, left)):
            return None
        return cache, row, wm, keep, (left, right, keep)

    def _rope_of_linear(self, rope, heads: int, hd: int):
        low = self.p._low.get(rope)
        if low is None or low[0] != "rope" or len(low[1]) != 2:
            return None
        x, pos = low[1]
        if tuple(x.shape) != (1, heads, 1, hd) or kind(x) != "reshape":
            return None
        lin = self.linears.get(x.inputs[0])
        if lin is None or not self.only_used_by(x, rope) or not self.only_used_by(lin.node, x):
            return None
        return lin, pos, x

    def attention_block(self, s):
        p = self.p
        q, kn, vn, mask = p._low[s][1]
        if len(q.shape) != 4 or q.shape[0] != 1 or q.shape[2] != 1:
            return None
        _, heads, _, hd = q.shape
        if len(kn.shape) != 4:
            return None
        _, kvh, ctx, hd2 = kn.shape
        if hd2 != hd or hd not in (32, 64, 128, 256) or heads % kvh:
            return None
        if tuple(mask.shape) != (1, 1, 1, ctx) or p.rdt(mask).name not in ("float32", "bfloat16", "float16"):
            return None
        if not self.only_used_by(q, s):
            return None
        rq = self._rope_of_linear(q, heads, hd)
        if rq is None:
            return None
        lin_q, pos, xq = rq
        kb = self._blend(kn, (1, kvh, ctx, hd))
        vb = self._blend(vn, (1, kvh, ctx, hd))
        if kb is None or vb is None or kb[2] is not vb[2]:
            return None
        kcache, krow, wm, kkeep, knodes = kb
        vcache, vrow, _, vkeep, vnodes = vb
        rk = self._rope_of_linear(krow, kvh, hd)
        if rk is None or rk[1] is not pos or not self.only_used_by(krow, knodes[1]):
            return None
        lin_k, _, xk = rk
        if kind(vrow) != "reshape" or tuple(vrow.shape) != (1, kvh, 1, hd):
            return None
        lin_v = self.linears.get(vrow.inputs[0])
        if lin_v is None or not self.only_used_by(vrow, vnodes[1]) or not self.only_used_by(lin_v.node, vrow):
            return None
        lins = [lin_q, lin_k, lin_v]
        if len({p.rdt(l.weight).str for l in lins}) != 1 or len({l.k for l in lins}) != 1:
            return None
        for cache_new in (kn, vn):
            if any(u is not s for u in self.uses(cache_new)):
                return None
        spec = self.input_spec(lins)
        if spec is None:
            return None
        claimed = [l.node for l in lins] + [xq, xk, vrow, q, krow, kn, vn, *knodes, *vnodes]
        p.claimed.update(claimed)
        self.claim_views(lins, spec)

        def emit() -> None:
            qkv = p.tmp((lin_q.n + lin_k.n + lin_v.n,), F32)
            self.emit_gemv(lins, spec, _lib.EPI_STORE, qkv)
            kview = self.cache_target(kcache, s)
            vview = self.cache_target(vcache, s)
            out = p.tmp(s.shape, F32)
            cos, sin, n_pos = p.rope_tables(q)
            splits = -(-ctx // 32)
            scratch = p.aux(shape=(splits * heads * (hd + 2),), dtype=np.float32)
            counters = p.aux(shape=(kvh,), dtype=np.int32, zero=True)  # used as unsigned
            p.add_step(
                "decode_attention", out,
                f"decode_attention(qkv={p._name(qkv)}, kv=({p._name(kview)}, {p._name(vview)}), "
                f"position, write_mask, mask, divisor={p._sdpa[s]!r})",
                qkv=qkv, q_off=0, k_off=lin_q.n, v_off=lin_q.n + lin_k.n,
                heads=heads, kv_heads=kvh, head_size=hd, context=ctx,
                position=p.contiguous(p.value(pos)), cos=cos, sin=sin, n_positions=n_pos,
                k_cache=kview, v_cache=vview, write_mask=p.contiguous(p.value(wm)),
                one_minus=p.rdt(kkeep), mask=p.contiguous(p.value(mask)), divisor=p._sdpa[s],
                scratch=scratch, counters=counters, flag=p.error_flag())
            p.set_value(s, out)
            p.set_value(kn, kview)
            p.set_value(vn, vview)
            for i, o in enumerate(p.outputs):
                if o is kn and kview.buf.kind == "input":
                    p.plan.aliases[i] = kcache
                if o is vn and vview.buf.kind == "input":
                    p.plan.aliases[i] = vcache

        self.units[s] = emit
        return claimed + [s]

    def cache_target(self, cache, sdpa) -> View:
        """The cache buffer updated in place, or a private copy when that is unsafe."""
        p = self.p
        view = p.value(cache)
        aliasable = (p.alias_caches and cache in p.dynamic and cache not in p.output_set
                     and len(self.uses(cache)) == 1 and view.is_contiguous())
        if aliasable:
            view.buf.bind = "pointer"
            return view
        out = p.tmp(cache.shape, view.dtype)
        p.add_step("copy", out, f"copy({p._name(view)})", src=view)
        return out

    # ------------------------------------------------------------ SwiGLU
    def swiglu(self, m):
        p = self.p
        a, b = m.inputs
        for gate_act, up in ((a, b), (b, a)):
            if not is_ew(gate_act, "div"):
                continue
            g, d = gate_act.inputs
            if not is_ew(d, "add") or not self.is_one(d.inputs[1]):
                continue
            e = d.inputs[0]
            if not is_ew(e, "exp") or not is_ew(e.inputs[0], "neg") or e.inputs[0].inputs[0] is not g:
                continue
            ng = e.inputs[0]
            lg, lu = self.linears.get(g), self.linears.get(up)
            if lg is None or lu is None or lg.k != lu.k or lg.n != lu.n:
                continue
            if p.rdt(lg.weight) != p.rdt(lu.weight):
                continue
            if not (self.only_used_by(g, ng, gate_act) and self.only_used_by(ng, e)
                    and self.only_used_by(e, d) and self.only_used_by(d, gate_act)
                    and self.only_used_by(gate_act, m) and self.only_used_by(up, m)):
                continue
            if any(p.rdt(n) != F32 for n in (ng, e, d, gate_act, m)):
                continue
            spec = self.input_spec([lg, lu])
            if spec is None:
                continue
            claimed = [g, up, ng, e, d, gate_act]
            p.claimed.update(claimed)
            self.claim_views([lg, lu], spec)

            def emit(lg=lg, lu=lu, spec=spec, m=m) -> None:
                out = p.tmp(m.shape, F32)
                self.emit_gemv([lg, lu], spec, _lib.EPI_SILU_MUL, out)
                p.set_value(m, out)

            self.units[m] = emit
            return claimed + [m]
        return None

    # ---------------------------------------------------------- residual
    def residual(self, add, done) -> None:
        p = self.p
        for lin_node, other in ((add.inputs[1], add.inputs[0]), (add.inputs[0], add.inputs[1])):
            lin = self.linears.get(lin_node)
            if lin is None or lin_node in done or lin_node in p.claimed:
                continue
            if not self.only_used_by(lin_node, add) or tuple(other.shape) != tuple(add.shape):
                continue
            if tuple(lin_node.shape) != tuple(add.shape) or p.rdt(add) != F32:
                continue
            if p.rdt(other).name not in ("float32", "bfloat16", "float16"):
                continue
            spec = self.input_spec([lin])
            if spec is None:
                continue
            p.claimed.add(lin_node)
            self.claim_views([lin], spec)
            if self.gathered_table(other) is not None:
                self.table_reads.add(add)

            def emit(lin=lin, spec=spec, add=add, other=other) -> None:
                out = p.tmp(add.shape, F32)
                self.emit_gemv([lin], spec, _lib.EPI_RESIDUAL, out, residual=other)
                p.set_value(add, out)

            self.units[add] = emit
            done.add(lin_node)
            return

    # ------------------------------------------------------------- plain
    def plain(self, lin: Linear) -> None:
        p = self.p
        spec = self.input_spec([lin])
        if spec is None:
            return
        self.claim_views([lin], spec)
        is_logits = lin.node in p.output_set and len(lin.node.shape) == 2

        def emit(lin=lin, spec=spec) -> None:
            out = p.tmp(lin.node.shape, F32)
            self.emit_gemv([lin], spec, _lib.EPI_ARGMAX if is_logits else _lib.EPI_STORE, out)
            p.set_value(lin.node, out)

        self.units[lin.node] = emit

    # -------------------------------------------------------------- emit
    def emit_gemv(self, lins: Sequence[Linear], spec, epilogue: int, out: View,
                  residual=None) -> None:
        p = self.p
        args: Dict[str, object] = dict(
            weights=[View.whole(p.plan.input_buffers[l.weight]) for l in lins],
            rows=[l.n for l in lins], k=lins[0].k, epilogue=epilogue)
        text = [f"w=[{', '.join(p.plan.input_buffers[l.weight].name for l in lins)}]"]
        if spec[0] == "norm":
            n = spec[1]
            x_node, w_node = p._low[n][1]
            rms = p._rms[n]
            args.update(norm=rms, norm_w=p.contiguous(p.value(w_node)))
            table = self.gathered_table(x_node)
            if table is not None:
                tab, ids = table
                args.update(x=View.whole(p.plan.input_buffers[tab]), x_index=p.contiguous(p.value(ids)),
                            norm_table=self.norm_table(tab, rms))
                text.append(f"x=rms_norm(gather({p.plan.input_buffers[tab].name}), table)")
            else:
                xv = p.contiguous(p.value(x_node))
                args.update(x=xv)
                text.append(f"x=rms_norm({p._name(xv)}, eps={rms.eps!r})")
        else:
            xv = p.contiguous(p.value(spec[1]))
            args.update(x=xv)
            text.append(f"x={p._name(xv)}")
        if residual is not None:
            table = self.gathered_table(residual)
            if table is not None and residual in p.claimed:
                tab, ids = table
                args.update(residual=View.whole(p.plan.input_buffers[tab]),
                            residual_index=p.contiguous(p.value(ids)))
                text.append(f"residual=gather({p.plan.input_buffers[tab].name})")
            else:
                rv = p.contiguous(p.value(residual))
                args.update(residual=rv)
                text.append(f"residual={p._name(rv)}")
        if "x_index" in args or "residual_index" in args:
            p.error_flag()  # out-of-range token ids are reported, not read
        if epilogue == _lib.EPI_ARGMAX:
            args.update(scratch_val=p.aux(shape=(2048,), dtype=np.float32),
                        scratch_idx=p.aux(shape=(2048,), dtype=np.int64),
                        counter=p.aux(shape=(1,), dtype=np.int32, zero=True),
                        argmax=p.aux(shape=(1,), dtype=np.int64, zero=True))
            for i, o in enumerate(p.outputs):
                if o is lins[0].node:
                    p.plan.argmax_of[i] = args["argmax"]
            text.append("argmax")
        names = {_lib.EPI_STORE: "store", _lib.EPI_RESIDUAL: "residual",
                 _lib.EPI_SILU_MUL: "silu_mul", _lib.EPI_ARGMAX: "argmax"}
        p.add_step("gemv", out, f"gemv_{names[epilogue]}({', '.join(text)})", **args)

    def gathered_table(self, node):
        """(table leaf, ids) when node = gather(constant table, single id)."""
        if kind(node) != "gather":
            return None
        tab, ids = node.inputs
        if tab.op is not None or tab in self.p.dynamic or not tab.cache_native:
            return None
        if int(np.prod(ids.shape)) != 1 or len(tab.shape) != 2:
            return None
        if self.p.rdt(ids).name not in ("int32", "int64"):
            return None
        return tab, ids

    def norm_table(self, table_leaf, rms):
        """Aux buffer of per-row norm sqrt terms, filled once at program build."""
        p = self.p
        key = (table_leaf, rms.divisor, rms.eps, tuple(d.str for d in rms.dts))
        if key in self._norm_tables:
            return self._norm_tables[key]
        rows = table_leaf.shape[0]
        buf = p.aux(shape=(rows,), dtype=np.float32)
        p.plan.init_steps.append(dict(name="rms_table", table=View.whole(p.plan.input_buffers[table_leaf]),
                                      spec=rms, out=buf))
        self._norm_tables[key] = buf
        return buf


def assign_prefetch(steps: Sequence) -> None:
    """Give each GEMV/attention step an L2 prefetch of an upcoming weight step.

    Walking the launch order, every prefetch-capable step prefetches the first
    not-yet-prefetched weight step among the next two, while the prefetched-
    but-unconsumed bytes stay under PREFETCH_OUTSTANDING.
    """
    weight_steps = [i for i, s in enumerate(steps) if s.name == "gemv"]
    nbytes = {i: sum(v.buf.size * v.dtype.itemsize for v in steps[i].args["weights"])
              for i in weight_steps}
    prefetched = set()
    for position, step in enumerate(steps):
        if step.name not in ("gemv", "decode_attention"):
            continue
        upcoming = [i for i in weight_steps if i > position][:2]
        consumed = {i for i in weight_steps if i <= position}
        outstanding = sum(min(nbytes[i], PREFETCH_CAP) for i in prefetched - consumed)
        for i in upcoming:
            if i in prefetched:
                continue
            size = min(nbytes[i], PREFETCH_CAP)
            if outstanding + size > PREFETCH_OUTSTANDING:
                break
            step.args["prefetch"] = (i, PREFETCH_CAP)
            prefetched.add(i)
            break
