"""The B200 decision readout: the hybrid backbone run level by level over packed tree levels, and the heads.

This is the drop-in for `HybridBackbone.encode_many` + `DecisionModel.forward` + `Worker.probabilities`
(janus/hybrid.py:1631-1807, janus/model.py:319-373, janus/server.py:277-282): the same packed requests in, the same
per-question logits and probabilities out. Per level and layer the work is: the dense projections (cuBLAS bf16
GEMMs on merged weights, as `_merge_projections` merges them, janus/hybrid.py:1108-1133) and every other op through
libjanus_b200 (janus_b200.ops): embedding + RMSNorm, residual add + RMSNorm (fp32 residual stream), the DeltaNet
prologue, the gated delta rule with the state fork read in place, the gated RMSNorm, attention q/k preparation,
tree attention with the output gate, the SwiGLU gate and the heads fused with the final norm. Levels keep their
DeltaNet states (conv tail, fp32 recurrent matrix) and attention keys/values only when a deeper level reads them.
"""

import dataclasses
import math

import numpy as np
import torch
import torch.nn.functional as F

from . import _lib, ops
from .config import LINEAR, ModelShape
from .plan import DevicePlan, build_levels, build_readout
from .prefix import PrefixSnapshot, stack_level0


class _Layer:
    pass


class DecisionReadout:
    """One model on one CUDA device. `weights`: name -> tensor (janus_b200.synthetic.make_weights layout, HF names),
    on any device; `mode`: "tree" (ScalarHead per leaf) or "listwise" (PointerHead). `ep`: a
    janus_b200.ep.ExpertParallel for MoE shapes served expert-parallel (this rank keeps only its experts; every rank
    of the group must run the same levels)."""

    def __init__(self, shape: ModelShape, weights, mode="tree", device="cuda", ep=None):
        if mode not in ("tree", "listwise"):
            raise ValueError("mode must be tree or listwise")
        self.shape, self.mode = shape, mode
        self.ep = ep if shape.moe else None
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("janus_b200 runs on CUDA devices only")
        dev = self.device
        w = lambda n, dt=torch.bfloat16: weights[n].to(dev, dt).contiguous()
        self.embed = w("embed_tokens.weight")
        self.final_norm = w("norm.weight")
        self.layers = []
        for i, kind in enumerate(shape.layer_types):
            p = f"layers.{i}."
            L = _Layer()
            L.kind = kind
            L.in_norm = w(p + "input_layernorm.weight")
            L.post_norm = w(p + "post_attention_layernorm.weight")
            if kind == LINEAR:
                a = p + "linear_attn."
                L.proj = torch.cat([w(a + n + ".weight") for n in ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a")])
                L.conv = w(a + "conv1d.weight").reshape(shape.conv_dim, shape.conv_kernel).contiguous()
                L.A_log, L.dt_bias, L.gnorm = w(a + "A_log"), w(a + "dt_bias"), w(a + "norm.weight")
                L.out = w(a + "out_proj.weight")
            else:
                a = p + "self_attn."
                L.qkv = torch.cat([w(a + n + ".weight") for n in ("q_proj", "k_proj", "v_proj")])
                L.q_norm, L.k_norm = w(a + "q_norm.weight"), w(a + "k_norm.weight")
                L.o = w(a + "o_proj.weight")
            m = p + "mlp."
            if shape.moe:
                L.router = w(m + "gate.weight")
                part = self.ep.shard if self.ep is not None else (lambda t: t)
                u8 = lambda n: part(weights[n]).to(dev).contiguous()
                bf = lambda n: part(weights[n]).to(dev, torch.bfloat16).contiguous()
                L.fp4 = (m + "experts.gate_up_proj.global") in weights
                if L.fp4:  # NVFP4 experts: e4m3 block scales (as bytes) and fp32 global scales per row
                    f8 = lambda n: part(weights[n]).to(dev).view(torch.uint8).contiguous()
                    f32 = lambda n: part(weights[n]).to(dev, torch.float32).contiguous()
                    L.gu_codes, L.gu_scales = u8(m + "experts.gate_up_proj"), f8(m + "experts.gate_up_proj.scales")
                    L.dn_codes, L.dn_scales = u8(m + "experts.down_proj"), f8(m + "experts.down_proj.scales")
                    L.gu_global, L.dn_global = f32(m + "experts.gate_up_proj.global"), f32(m + "experts.down_proj.global")
                else:
                    L.gu_codes, L.gu_scales = u8(m + "experts.gate_up_proj"), bf(m + "experts.gate_up_proj.scales")
                    L.dn_codes, L.dn_scales = u8(m + "experts.down_proj"), bf(m + "experts.down_proj.scales")
                # the shared expert's gate/up rows in the order of the tcgen05 GEMM's SwiGLU epilogue
                L.shared_gate_up = ops.swiglu_weight(w(m + "shared_expert.gate_proj.weight"),
                                                     w(m + "shared_expert.up_proj.weight"))
                L.shared_down = w(m + "shared_expert.down_proj.weight")
                L.shared_gate = w(m + "shared_expert_gate.weight")
            else:
                gate, up = w(m + "gate_proj.weight"), w(m + "up_proj.weight")
                if gate.shape[0] % 128 == 0:  # the tcgen05 GEMM's SwiGLU epilogue takes 128-row gate/up blocks
                    L.gate_up, L.gate_up_swiglu = None, ops.swiglu_weight(gate, up)
                else:
                    L.gate_up, L.gate_up_swiglu = torch.cat([gate, up]), None
                del gate, up
                L.down = w(m + "down_proj.weight")
            self.layers.append(L)
        f32 = lambda n: w(n, torch.float32)
        self.head = {k[5:]: f32(k) for k in weights if k.startswith("head.")}
        r = shape.rotary_dim
        # Qwen3_5TextRotaryEmbedding.compute_default_rope_parameters, fp32
        self.inv_freq = (1.0 / (shape.rope_theta ** (torch.arange(0, r, 2, dtype=torch.int64).float() / r))).to(dev)
        self.group = shape.heads // shape.kv_heads
        self.tile_tokens = ops.tree_attention_tile_tokens(shape.head_dim, shape.heads, shape.kv_heads)
        self.last_plan = None
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)  # set by a device-side wait that ran out

    # ------------------------------------------------------------------------------------------------ level pass

    def _level(self, lv, plan, history, logits):
        s = self.shape
        d, T = lv.depth, lv.T
        eps = s.rms_eps
        rs, rot = plan[(d, "row_start")], plan[(d, "row_of_token")]
        x, y = ops.embed_rmsnorm(self.embed, plan[(d, "ids")], self.layers[0].in_norm, eps)
        pending = None
        kept = []
        Vd, C = s.value_dim, s.conv_dim
        for i, L in enumerate(self.layers):
            if i > 0:
                y = ops.add_rmsnorm(x, pending, L.in_norm, eps)
            if L.kind == LINEAR:
                proj = F.linear(y, L.proj)
                parent_state = history[d - 1][i] if d > 0 else (None, None)
                q, k, v, g, beta, tail = ops.gdn_prologue(
                    proj, rs, rot, plan[(d, "parent")] if d > 0 else None, parent_state[0], lv.keep, L.conv, L.A_log,
                    L.dt_bias, s.lin_k_heads, s.lin_k_dim, s.lin_v_heads, s.lin_v_dim)
                if self._chunked(lv):
                    o, S = ops.gdn_chunk_scan(q, k, v, g, beta, rs, plan[(d, "chunk_start")], int(lv.chunk_start[-1]),
                                              parent_state[1], plan[(d, "parent")] if d > 0 else None, lv.keep,
                                              1.0 / math.sqrt(s.lin_k_dim), status=self.status)
                elif self._packed_fork(lv):
                    fc_parent = plan[(d, "fc_parent")]
                    o, S = ops.gdn_chunk_scan(q, k, v, g, beta, plan[(d, "fc_start")], plan[(d, "fc_chunks")],
                                              int(fc_parent.numel()), parent_state[1], fc_parent, False,
                                              1.0 / math.sqrt(s.lin_k_dim), status=self.status, segment=rot)
                else:
                    o, S = ops.gdn_fork_recurrent(q, k, v, g, beta, rs, plan[(d, "child_start")], parent_state[1],
                                                  lv.keep, 1.0 / math.sqrt(s.lin_k_dim))
                core = ops.gated_rmsnorm(o, proj[:, C:C + Vd], L.gnorm, eps)
                h = F.linear(core, L.out)
                kept.append((tail, S) if lv.keep else None)
            else:
                qkv = F.linear(y, L.qkv)
                D, Hq, Hkv = s.head_dim, s.heads, s.kv_heads
                q, kk, vv = ops.attn_qk_prep(qkv, plan[(d, "pos")], self.inv_freq, L.q_norm, L.k_norm, eps, Hq, Hkv, D)
                keys = [history[l][i][0] for l in range(d)] + [kk]
                values = [history[l][i][1] for l in range(d)] + [vv]
                gate = qkv[:, :Hq * 2 * D].view(T, Hq, 2 * D)[:, :, D:]
                o = ops.tree_attention(q, keys, values, [plan[(d, "lo", l)] for l in range(d)],
                                       [plan[(d, "hi", l)] for l in range(d)], rs, rot,
                                       plan[(d, "tiles", self.tile_tokens)].view(-1, 2), gate, D ** -0.5,
                                       status=self.status)
                h = F.linear(o, L.o)
                kept.append((kk, vv) if lv.keep else None)
            y = ops.add_rmsnorm(x, h, L.post_norm, eps)
            pending = self._moe(y, L) if s.moe else F.linear(self._swiglu(y, L), L.down)
        ops.add_rmsnorm(x, pending, self.final_norm, eps)  # the last residual add (its normed output is unused)
        self._heads(d, x, plan, logits)
        return kept

    def _swiglu(self, y, L):
        """The dense MLP's silu(gate(y)) * up(y) (`_silu_mul`, janus/hybrid.py:263): one tcgen05 GEMM whose epilogue
        applies the SwiGLU to the fp32 accumulators and writes the I-wide product once; widths that are not multiples
        of 128 take the merged GEMM and the silu_mul kernel."""
        if L.gate_up_swiglu is not None:
            return ops.gemm_bf16(y, L.gate_up_swiglu, swiglu=True, status=self.status)
        return ops.silu_mul(F.linear(y, L.gate_up))

    def _moe(self, y, L):
        """Qwen3_5MoeSparseMoeBlock (transformers qwen3_5_moe :773-791) on the W4A16 experts: router logits in fp32
        (bf16 GEMM, fp32 output) -> routing plan -> gate_up grouped GEMM (silu(gate) * up) -> down grouped GEMM times
        the routing weight -> per-token sum plus the sigmoid-gated shared expert."""
        k = self.shape.top_k
        if L.router.shape[0] <= 256 and k in (1, 2, 4, 6, 8):
            # the router GEMM, its softmax / top-k and the shared expert's gate logit in one tensor-core pass
            plan, sg = ops.moe_route_fused(y, L.router, k, w_gate=L.shared_gate, status=self.status)
        else:
            plan = ops.moe_route(torch.mm(y, L.router.t(), out_dtype=torch.float32), k)
            sg = torch.mm(y, L.shared_gate.t(), out_dtype=torch.float32).reshape(-1)
        if self.ep is not None:
            return self._moe_ep(y, L, plan[0], plan[1], sg)
        h = self._experts(y, L, plan, True, k)
        y2 = self._experts(h, L, plan, False, k, topk_w=plan[1])
        shared = self._shared_expert(y, L)
        return ops.moe_combine(y2, k, shared, sg)

    def _shared_expert(self, y, L):
        """The shared expert's SwiGLU (transformers qwen3_5_moe :778-791) on the tcgen05 GEMM: gate/up with the SwiGLU
        epilogue (silu(gate) * up from the fp32 accumulators, rounded once), then the down projection."""
        return ops.gemm_bf16(ops.gemm_bf16(y, L.shared_gate_up, swiglu=True, status=self.status), L.shared_down,
                             status=self.status)

    def _moe_ep(self, y, L, topk_idx, topk_w, sg):
        """The expert-parallel MoE block (janus_b200/ep.py): dispatch rows to the ranks owning their experts, grouped
        GEMMs over this rank's experts, fp32 partial per received row, combine on the owner with the shared expert."""
        k, ep = self.shape.top_k, self.ep
        if ep.static:  # fixed shapes, no host read: the capturable exchange, blocks of the level's agreed capacity
            (rows, slot_e, slot_w), handle = ep.dispatch_static(y, topk_idx, topk_w, self._ep_capacity)
        else:
            (rows, slot_e, slot_w), handle = ep.dispatch(y, topk_idx, topk_w)
        H = y.shape[1]
        if rows.shape[0]:
            plan = ops.moe_plan(slot_e, ep.local)
            h = self._experts(rows, L, plan, True, k)
            y2 = self._experts(h, L, plan, False, k, topk_w=slot_w.reshape(-1))
            part = ops.moe_reduce_slots(y2, k, slot_e)
        else:
            part = torch.empty(0, H, dtype=torch.float32, device=y.device)
        shared = self._shared_expert(y, L)
        back, row_index = ep.combine_static(part, handle) if ep.static else ep.combine(part, handle)
        return ops.moe_combine_ep(back, row_index, shared, sg)

    def _experts(self, x, L, plan, gated, k, topk_w=None):
        """One grouped GEMM over the layer's experts in their stored format (int4 group 128, or NVFP4)."""
        if L.fp4:
            codes, bs, gs = (L.gu_codes, L.gu_scales, L.gu_global) if gated else (L.dn_codes, L.dn_scales, L.dn_global)
            return ops.moe_grouped_nvfp4(x, codes, bs, gs, plan, gated, k, topk_w=topk_w, status=self.status)
        codes, sc = (L.gu_codes, L.gu_scales) if gated else (L.dn_codes, L.dn_scales)
        return ops.moe_grouped_w4a16(x, codes, sc, plan, gated, k, topk_w=topk_w, status=self.status)

    CHUNK_MIN_TOKENS = 32  # mean row length from which a level runs the chunked rule (rows are read once per chunk)

    def _chunked(self, lv):
        """The chunked rule for levels of long rows (tensor-core WY form), the fork-recurrent rule for short ones
        (the reference's split at janus/hybrid.py:115-118, RECURRENT_TOKENS = 16)."""
        s = self.shape
        return s.lin_k_dim == 128 and s.lin_v_dim == 128 and lv.T >= self.CHUNK_MIN_TOKENS * lv.B

    def _packed_fork(self, lv):
        """Short sibling rows that keep no state run as the segmented chunk scan: their tokens packed into 64-token
        runs per parent, each row starting from the parent's state (tensor cores instead of a token-by-token walk)."""
        s = self.shape
        return (s.lin_k_dim == 128 and s.lin_v_dim == 128 and lv.depth > 0 and not lv.keep
                and lv.fork_chunks() is not None)

    def _heads(self, d, x, plan, logits):
        """The readout rows of level d through the head, their logits scattered to their slots (row and slot tables
        come with the level plan: no host data enters the device pass)."""
        ro = self._readout
        hd, s = self.head, self.shape
        if d in ro.scalar:
            z = ops.head_scalar(x, plan[(d, "scalar_rows")], self.final_norm, s.rms_eps, hd["norm.weight"],
                                hd["norm.bias"], 1e-5, hd["out.weight"].reshape(-1), hd["out.bias"])
            logits.index_copy_(0, plan[(d, "scalar_slots")].long(), z)
        if d in ro.pointer:
            z = ops.head_pointer(x, plan[(d, "opt_rows")], plan[(d, "opt_q")], plan[(d, "dec_rows")], self.final_norm,
                                 s.rms_eps, hd["norm.weight"], hd["norm.bias"], 1e-5, hd["query.weight"],
                                 hd["key.weight"])
            logits.index_copy_(0, plan[(d, "pointer_slots")].long(), z)

    # ------------------------------------------------------------------------------------------------ public API

    def plan(self, packs):
        for p in packs:
            ids = p.input_ids
            if ids.numel() and (int(ids.min()) < 0 or int(ids.max()) >= self.shape.vocab):
                raise ValueError(f"token ids must lie in [0, {self.shape.vocab})")
        levels, index = build_levels(packs)
        readout = build_readout(packs, levels, index, self.mode)
        return levels, readout

    def prepare(self, packs, prefixes=None):
        """Host planning plus the one host-to-device copy of the level tables: (levels, readout, device plan).

        `prefixes` (parallel to `packs`, as `HybridBackbone.encode_many(prefixes=...)`, janus/hybrid.py:1648-1659):
        per pack a PrefixSnapshot of its state (`encode_prefixes`) or None. The state level then runs only for the
        packs without one (as one batch), every snapshot is checked against its pack's state tokens, and the pass
        starts at level 1 from the snapshots stacked in pack order."""
        levels, readout = self.plan(packs)
        plan = DevicePlan(levels, readout, self.device, tile_tokens=(self.tile_tokens,))
        plan.prefix_history = None if prefixes is None else self._prefix_history(packs, levels, readout, prefixes)
        if self.ep is not None and self.ep.static:  # the static exchange's block size per level, agreed by the group
            plan.ep_capacity = {lv.depth: self.ep.agree_capacity(lv.T, self.device) for lv in levels}
        return levels, readout, plan

    def encode_prefixes(self, packs):
        """HybridBackbone.encode_prefixes (janus/hybrid.py:1641-1646): the state level of several packs as one
        batch, one PrefixSnapshot per pack (conv tails and recurrent states of the DeltaNet layers, keys and values
        of the attention layers after the state's last token), copied out of the level batch so it outlives the
        call. Raises if a device-side wait of the pass ran out."""
        levels, readout = self.plan(packs)
        lv = levels[0] if levels else None
        self._check_state_rows(lv, len(packs))
        plan = DevicePlan(levels[:1], readout, self.device, tile_tokens=(self.tile_tokens,))
        self._readout = readout
        logits = torch.zeros(readout.n_slots, dtype=torch.float32, device=self.device)
        self.status.zero_()
        self._ep_capacity = (self.ep.agree_capacity(lv.T, self.device)
                             if self.ep is not None and self.ep.static else None)
        kept = self._level(dataclasses.replace(lv, keep=True), plan, [], logits)
        self.check_status()
        attention = [L.kind != LINEAR for L in self.layers]
        snaps = []
        for r in range(len(packs)):
            a, b = int(lv.row_start[r]), int(lv.row_start[r + 1])
            states = [(first[a:b].clone(), second[a:b].clone()) if att else (first[r].clone(), second[r].clone())
                      for att, (first, second) in zip(attention, kept)]
            snaps.append(PrefixSnapshot(states, attention, lv.ids[a:b]))
        return snaps

    @staticmethod
    def _check_state_rows(lv, n_packs):
        if lv is None or lv.B != n_packs or any(int(row[0]) != r for r, row in enumerate(lv.rows)):
            raise ValueError("prefix snapshots need one state segment per pack at level 0")

    def _prefix_history(self, packs, levels, readout, prefixes):
        if len(prefixes) != len(packs):
            raise ValueError(f"{len(prefixes)} prefixes for {len(packs)} packs")
        if 0 in readout.scalar or 0 in readout.pointer:
            raise ValueError("a pack reads out at its state level, which a snapshot skips")
        lv = levels[0] if levels else None
        self._check_state_rows(lv, len(packs))
        snaps = list(prefixes)
        missing = [i for i, s in enumerate(snaps) if s is None]
        if missing:
            for i, s in zip(missing, self.encode_prefixes([packs[i] for i in missing])):
                snaps[i] = s
        attention = [L.kind != LINEAR for L in self.layers]
        for r, s in enumerate(snaps):
            a, b = int(lv.row_start[r]), int(lv.row_start[r + 1])
            if not isinstance(s, PrefixSnapshot) or s.attention != attention:
                raise ValueError(f"pack {r}: not a snapshot of this model's layers")
            if s.tokens != b - a or not np.array_equal(s.ids, lv.ids[a:b]):
                raise ValueError(f"pack {r}: the snapshot is of another state")
            dev = s.device
            if dev is None or dev.type != "cuda" or (self.device.index is not None and dev.index != self.device.index):
                raise ValueError(f"pack {r}: the snapshot lives on {dev}, the model on {self.device}")
        return stack_level0(snaps, attention)

    def run(self, prepared):
        """The device pass over prepared levels: all option logits as one fp32 device tensor [slots]."""
        levels, readout, plan = prepared
        self._readout = readout
        self.last_plan = plan
        logits = torch.zeros(readout.n_slots, dtype=torch.float32, device=self.device)
        self.status.zero_()
        history = []
        prefix = getattr(plan, "prefix_history", None)
        if prefix is not None:  # every pack's state level comes from a snapshot: start at level 1
            history.append(prefix)
        for lv in levels[len(history):]:
            self._ep_capacity = getattr(plan, "ep_capacity", {}).get(lv.depth)
            history.append(self._level(lv, plan, history, logits))
        return logits

    def logits_flat(self, packs, prefixes=None):
        """All option logits of a batch as one fp32 device tensor [slots] (order: pack, question, option; the
        constant false option of a tree-mode noul has no slot) plus the host readout layout. `prefixes`: per pack
        a PrefixSnapshot of its state or None (see `prepare`)."""
        prepared = self.prepare(packs, prefixes)
        return self.run(prepared), prepared[1]

    def check_status(self):
        """Raise if a bounded device-side wait of the last run ran out (its results are then invalid)."""
        if int(self.status.item()) != 0:
            raise _lib.JanusError("a device-side wait (tree attention or chunk scan) ran out; the results of this run "
                                  "are invalid")

    def forward_many(self, packs, prefixes=None):
        """Per pack, per question, the logits as fp32 CPU tensors (janus/model.py:368-373 + :319-366)."""
        flat, readout = self.logits_flat(packs, prefixes)
        host = flat.cpu()
        self.check_status()
        return assemble(host, readout)

    def probabilities(self, packs, temperatures=None, prefixes=None):
        """Worker.probabilities (janus/server.py:277-282): softmax(logits / T) per question, T = 1 by default."""
        out = []
        for i, per in enumerate(self.forward_many(packs, prefixes)):
            ts = (temperatures[i] if temperatures else None) or [1.0] * len(per)
            out.append([torch.softmax(z / t, dim=-1) for z, t in zip(per, ts)])
        return out


def assemble(host_logits, readout):
    """Per pack, per question logits (fp32 CPU tensors) from the flat host tensor and the readout layout; a slot of
    None (the false option of a tree-mode noul) is the constant 0."""
    flat = np.append(host_logits.numpy().astype(np.float32, copy=False), np.float32(0.0))  # index -1: the constant 0
    res = []
    for layout in readout.layout:
        res.append([torch.from_numpy(flat[np.array([-1 if s is None else s for s in slots], dtype=np.int64)])
                    for slots in layout])
    return res
