"""Expert parallelism for the W4A16 MoE blocks of the A3B shape over the ranks of one process group.

The reference serves on one device (janus/server.py:157: "the upgrade path is one Worker per device") and has no
collective anywhere; this is the partition its MoE shape needs at 8 GPUs. Every rank runs its own requests through
attention and DeltaNet (data parallel) and holds the router, the shared expert and 1/W of the routed experts
(experts [rank*E/W, (rank+1)*E/W)). Per MoE layer:

1. route locally (router softmax, top-k, renormalise: janus_b200_moe_route);
2. dispatch: each token row goes once to every rank that owns at least one of its k experts (deduplicated per
   rank, not per expert), with its k (local expert id or -1, routing weight) slots; counts first, then rows and
   slots, all with NCCL all_to_all_single (rows land in this GPU's memory; no kernel reads a peer's memory);
3. the receiving rank runs the grouped W4A16 GEMMs over the received rows (plan from the explicit local expert
   ids: janus_b200_moe_plan) and reduces each row's local slots to one fp32 partial (janus_b200_moe_reduce_slots);
4. combine: the fp32 partials go back to the owner (the reverse all_to_all), which adds them in rank order plus
   the gated shared expert and rounds once to bf16 (janus_b200_moe_combine_ep).

The fp32 partials keep the reference's fp32 sum over the k experts (janus/moe_w4a16.py:140); only the order of
that sum changes (per rank, then over ranks). In the default form the split sizes of the row all_to_all are read on
the host (one small device-to-host copy per layer), so it sends exactly the rows needed but is not CUDA-graph
capturable. `ExpertParallel(..., static=True)` is the capturable form: fixed shapes, no host read and two
collectives per layer (section `dispatch_static`), at the price of fixed-size blocks (each destination's block is
as large as the rank's token count). Every rank must run the same sequence of MoE layers (same levels), as all its
collectives pair up by order.
"""

import torch
import torch.distributed as dist


class ExpertParallel:
    """The expert partition of one process group and the dispatch / combine exchanges of a MoE layer."""

    def __init__(self, n_experts, group=None, static=False):
        self.group = group
        self.static = static
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if n_experts % self.world:
            raise ValueError(f"{n_experts} experts do not split over {self.world} ranks")
        self.n_experts = n_experts
        self.local = n_experts // self.world
        self.first = self.rank * self.local

    def shard(self, experts):
        """This rank's experts of a tensor with the expert index first ([E, ...])."""
        if experts.shape[0] != self.n_experts:
            raise ValueError(f"expected {self.n_experts} experts, got {experts.shape[0]}")
        return experts[self.first:self.first + self.local].contiguous()

    def _a2a(self, out, inp, out_splits, in_splits):
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)
        return out

    def dispatch(self, x, topk_idx, topk_w):
        """x [S, H]; topk_idx [S, k] global expert ids; topk_w [S, k] fp32 ->
        ((rows [R, H], slot_expert int32 [R, k] local ids or -1, slot_w fp32 [R, k]), handle for combine)."""
        S, k = topk_idx.shape
        W, L, dev = self.world, self.local, x.device
        dest = torch.div(topk_idx.long(), L, rounding_mode="floor")  # owning rank of every slot
        hit = torch.zeros(S, W, dtype=torch.bool, device=dev)
        if S:
            hit.scatter_(1, dest, True)
        send_rank, send_tok = hit.t().nonzero(as_tuple=True)  # by destination rank, then token order
        send_counts = hit.sum(0).to(torch.int64)
        mine = dest.index_select(0, send_tok) == send_rank[:, None]
        local_id = topk_idx.long().index_select(0, send_tok) - send_rank[:, None] * L
        slot_e = torch.where(mine, local_id, torch.full_like(local_id, -1)).to(torch.int32)
        slot_w = topk_w.index_select(0, send_tok).float().contiguous()
        rows = x.index_select(0, send_tok).contiguous()
        recv_counts = torch.empty_like(send_counts)
        self._a2a(recv_counts, send_counts, None, None)
        sc, rc = send_counts.tolist(), recv_counts.tolist()
        R = sum(rc)
        recv_rows = self._a2a(x.new_empty(R, x.shape[1]), rows, rc, sc)
        recv_e = self._a2a(torch.empty(R, k, dtype=torch.int32, device=dev), slot_e, rc, sc)
        recv_w = self._a2a(torch.empty(R, k, dtype=torch.float32, device=dev), slot_w, rc, sc)
        row_index = torch.full((S, W), -1, dtype=torch.int32, device=dev)
        row_index[send_tok, send_rank] = torch.arange(send_tok.numel(), dtype=torch.int32, device=dev)
        return (recv_rows, recv_e, recv_w), (sc, rc, row_index)

    def dispatch_static(self, x, topk_idx, topk_w, capacity):
        """The capturable dispatch: one all_to_all_single with equal splits, no host read. Destination d gets a block
        of `capacity` rows (the same on every rank and at least every rank's token count S: the level's graph bucket
        agrees on it beforehand, `agree_capacity`); a row carries the token's H values and its k (local expert id or
        -1, routing weight) slots as raw bits beside them, so rows and slots travel together. A token's row goes to
        row `pos` of block d, pos counting this rank's earlier tokens that also go to d (a device cumulative sum);
        unused rows carry only -1 slots, so the receiver's grouped GEMMs skip them.
        Returns ((rows [W*C, H] view in x's dtype, slot_expert int32 [W*C, k], slot_w fp32 [W*C, k]), row_index
        int32 [S, W]: where each token's row sits in the blocks, -1 where it is not sent)."""
        S, k = topk_idx.shape
        W, L, dev, H, C = self.world, self.local, x.device, x.shape[1], int(capacity)
        if S > C:
            raise ValueError(f"{S} tokens exceed the agreed capacity {C}")
        raw = {2: torch.int16, 4: torch.int32}[x.element_size()]
        meta = 8 * k // x.element_size()  # k int32 ids + k fp32 weights, in units of x's element size
        dest = torch.div(topk_idx.long(), L, rounding_mode="floor")
        hit = torch.zeros(S, W, dtype=torch.bool, device=dev)
        if S:
            hit.scatter_(1, dest, True)
        pos = torch.cumsum(hit.to(torch.int64), 0) - 1
        block = torch.arange(W, device=dev, dtype=torch.int64)[None, :] * C
        flat = torch.where(hit, block + pos, torch.full_like(pos, W * C))  # W * C: a scratch row for non-hits
        buf = torch.empty(W * C + 1, H + meta, dtype=raw, device=dev)
        rows = buf[:, :H].view(x.dtype)
        ids = buf[:, H:H + meta // 2].view(torch.int32)
        wts = buf[:, H + meta // 2:].view(torch.float32)
        ids.fill_(-1)
        local_id = (topk_idx.long() - dest * L).to(torch.int32)
        w32 = topk_w.float()
        for d in range(W):
            idx = flat[:, d]
            rows.index_copy_(0, idx, x)
            ids.index_copy_(0, idx, torch.where(dest == d, local_id, torch.full_like(local_id, -1)))
            wts.index_copy_(0, idx, w32)
        recv = torch.empty(W * C, H + meta, dtype=raw, device=dev)
        # as bytes: NCCL has no 16-bit integer type (the rows are raw bits either way)
        dist.all_to_all_single(recv.view(torch.uint8), buf[:W * C].view(torch.uint8), group=self.group)
        row_index = torch.where(hit, flat, torch.full_like(flat, -1)).to(torch.int32)
        return ((recv[:, :H].view(x.dtype), recv[:, H:H + meta // 2].view(torch.int32).contiguous(),
                 recv[:, H + meta // 2:].view(torch.float32).contiguous()), row_index)

    def agree_capacity(self, tokens, device):
        """The block size of the static exchange for a level: the largest token count over the group's ranks (one
        small all_reduce, on the host side of the pass: at planning time, before a captured level runs)."""
        t = torch.tensor([int(tokens)], dtype=torch.int64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        return int(t.item())

    def combine_static(self, partials, row_index):
        """partials fp32 [W*S, H] in the received blocks' order -> (the owner's partials fp32 [W*S, H] in the order it
        sent them, row_index [S, W]): one all_to_all_single with equal splits."""
        back = torch.empty_like(partials)
        dist.all_to_all_single(back, partials.contiguous(), group=self.group)
        return back, row_index

    def combine(self, partials, handle):
        """partials fp32 [R, H] of the received rows -> (the owner's partials fp32 [n_sent, H], row_index [S, W])."""
        sc, rc, row_index = handle
        back = partials.new_empty(sum(sc), partials.shape[1])
        self._a2a(back, partials.contiguous(), sc, rc)
        return back, row_index


def sum_partials(back, row_index):
    """The owner's sum of the per-rank partials in rank order (fp32 [S, H]); the torch statement of what
    janus_b200_moe_combine_ep computes before it adds the shared expert."""
    S, W = row_index.shape
    out = torch.zeros(S, back.shape[1], dtype=torch.float32, device=back.device)
    for w in range(W):
        idx = row_index[:, w].long()
        has = idx >= 0
        out[has] += back[idx[has]]
    return out
