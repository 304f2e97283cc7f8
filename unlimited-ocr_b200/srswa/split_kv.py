"""Split-KV decode of one long sequence over the ranks of a process group.

The 1M-token decode (16384 blocks of 64 tokens per layer) keeps K/V, the
index keys and the block summaries k_bar of a contiguous range of blocks on
each GPU; the GPU owning the newest blocks also owns the local window.  One
decode step of one layer is:

1. every rank scores the blocks it owns and keeps its best M as packed keys
   (``srswa_route_shard_keys``);
2. all-gather of the ``[world, rows, M]`` keys (8 bytes each);
3. every rank merges them into the same global selection
   (``srswa_route_merge_keys``: exact top-M, entmax, top-K, bias; the top-M of
   the whole row lies inside the union of the ranks' top-Ms) and keeps the
   slots it owns;
4. every rank attends its own selected blocks, the window owner also the
   window (``srswa_decode_attend`` with ``skip_local`` elsewhere), giving a
   partial output (fp32) and its log-sum-exp (``-inf`` when empty);
5. all-gather of the partials (o and its log-sum-exp packed in one buffer)
   and the log-sum-exp merge (``srswa_lse_merge``).

Every rank issues the same two collectives in the same order on every step.
The reference decodes one GPU at a time (``_dash_decode_forward``,
hf-model-code/modeling_deepseekv2.py:483-530); the selection it must
reproduce is ``_block_scores_infer`` + ``_infer_route_select`` (:339-430) and
the attention ``_decode_attend`` (:455-481).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class ShardPlan:
    """Contiguous block ranges per rank: ranks 0..world-2 own ``per`` blocks
    of the first ``nblk_filled``; the last rank owns the rest, including the
    blocks the sequence grows into, so the window (the newest blocks) stays on
    one rank."""

    nblk_total: int
    world: int
    rank: int
    nblk_filled: int

    @property
    def per(self) -> int:
        return max(1, math.ceil(self.nblk_filled / self.world))

    def bounds(self, r: int) -> tuple[int, int]:
        lo = min(r * self.per, self.nblk_total)
        hi = self.nblk_total if r == self.world - 1 else min((r + 1) * self.per, self.nblk_total)
        return lo, hi

    @property
    def lo(self) -> int:
        return self.bounds(self.rank)[0]

    @property
    def hi(self) -> int:
        return self.bounds(self.rank)[1]

    def owner(self, blk: int) -> int:
        for r in range(self.world):
            lo, hi = self.bounds(r)
            if lo <= blk < hi:
                return r
        raise ValueError(f"block {blk} outside [0, {self.nblk_total})")


class CudaBackend:
    """The library's kernels on the current CUDA device, NCCL collectives."""

    def __init__(self, group=None):
        from . import ops
        self.ops = ops
        self.group = group

    def shard_keys(self, idx_q, layer, plan, q_pos, rp):
        return self.ops.route_shard_keys(
            idx_q, layer["kbar"], block_offset=plan.lo, nblk_local=plan.hi - plan.lo,
            nblk_total=plan.nblk_total, q_pos=q_pos, rows_per_seq=idx_q.shape[0],
            block_table=layer.get("kbar_table"), **rp)

    def merge_keys(self, keys, plan, rp):
        p = {k: v for k, v in rp.items() if k not in ("block_size", "local_blocks")}
        return self.ops.route_merge_keys(keys, nblk_total=plan.nblk_total, own=(plan.lo, plan.hi),
                                         want=("topi32", "bias"), **p)

    def select(self, idx_q, layer, plan, q_pos, rp):
        """The merged selection of the whole row (topi32, bias, topi32_own):
        one launch on a single rank, else shard keys -> all-gather -> merge."""
        if plan.world == 1:
            return self._shard_select(idx_q, layer, plan, q_pos, rp, None)
        keys = self.shard_keys(idx_q, layer, plan, q_pos, rp)               # [N, M]
        return self.merge_keys(self.gather_keys(keys, plan.world), plan, rp)

    def _shard_select(self, idx_q, layer, plan, q_pos, rp, exchange):
        return self.ops.route_shard_select(
            idx_q, layer["kbar"], block_offset=plan.lo, nblk_local=plan.hi - plan.lo, nblk_total=plan.nblk_total,
            q_pos=q_pos, rows_per_seq=idx_q.shape[0], block_table=layer.get("kbar_table"),
            own=(plan.lo, plan.hi), want=("topi32", "bias"), exchange=exchange, **rp)

    def attend(self, q, layer, topi, bias, q_pos, *, block_size, local_blocks, sm_scale, skip_local,
               out_dtype=torch.float32):
        N, H, D = q.shape
        if out_dtype == torch.float32:
            # partial o and its lse packed in one buffer (padded to 16 bytes):
            # one all-gather moves both
            buf = torch.empty(-(-(N * H * D + N * H) // 4) * 4, device=q.device, dtype=torch.float32)
            out, lse = buf[:N * H * D].view(N, H, D), buf[N * H * D:N * H * D + N * H].view(N, H)
        else:
            out, lse = torch.empty(q.shape, device=q.device, dtype=out_dtype), None
        # overlap: the attend follows the router's last kernel on the stream and
        # starts on the window keys (q and the caches predate the router)
        return self.ops.decode_attend(q, layer["k_cache"], layer["v_cache"], topi, bias, block_size=block_size,
                                      local_blocks=local_blocks, sm_scale=sm_scale, out=out,
                                      block_table=layer["block_table"], q_pos=q_pos, rows_per_req=N,
                                      lse=True, skip_local=skip_local, lse_out=lse, overlap=True)

    def gather_keys(self, keys, world):
        """All-gather of the router keys [N, M] -> [world, N, M]."""
        return self.all_gather(keys, world)

    def exchange_partials(self, o_part, lse_part, world):
        """All-gather of the packed partials -> ([world,N,H,D], [world,N,H]) views."""
        N, H, D = o_part.shape
        n = N * H * D + N * H
        buf = torch.as_strided(o_part, (-(-n // 4) * 4,), (1,))   # the packed buffer of attend()
        g = self.gather_partials(buf, world)
        return g[:, :N * H * D].view(world, N, H, D), g[:, N * H * D:n].view(world, N, H)

    def gather_partials(self, buf, world):
        return self.all_gather(buf, world)

    def lse_merge(self, o_parts, lse_parts, out_dtype):
        return self.ops.lse_merge(o_parts, lse_parts, out_dtype=out_dtype)[0]

    def all_gather(self, x, world):
        if world == 1:
            return x.unsqueeze(0)
        import torch.distributed as dist
        out = torch.empty((world,) + tuple(x.shape), device=x.device, dtype=x.dtype)
        dist.all_gather_into_tensor(out, x.contiguous(), group=self.group)
        return out


class PeerBackend(CudaBackend):
    """CudaBackend whose two exchanges per layer go through peer memory
    (srswa.peer.PeerAllGather over CUDA IPC) instead of a library all-gather,
    with no collective after set-up.  One object serves every layer of a
    step (the two regions alternate, which keeps a rank from overwriting
    data a peer still reads).  rows / topm / heads / head_dim bound the
    payloads.  mode:

    * "ll" (default): the router's one-launch select exchanges the keys and
      the attend stores its partials as LL words (payload + epoch in one
      8-byte store, no fence or flag); the log-sum-exp merge polls them;
    * "flag": the same kernels with the flag protocol (payload stores, a
      system-scope fence, then a released flag per source);
    * "launch": each exchange is its own push launch + wait launch."""

    MODES = ("ll", "flag", "launch")

    def __init__(self, group=None, *, rows, topm, heads, head_dim, mode="ll"):
        super().__init__(group)
        from .peer import PeerAllGather
        if mode not in self.MODES:
            raise ValueError(f"mode {mode!r} not in {self.MODES}")
        self.mode = mode
        self.fused = mode != "launch"
        ll = mode == "ll"
        words = 2 if ll else 1       # LL: 8 bytes per 32-bit payload word
        self.keys_x = PeerAllGather(rows * topm * 8 * words, group, ll=ll)
        self.part_x = PeerAllGather(-(-(rows * heads * head_dim + rows * heads) // 4) * 16 * words, group, ll=ll)

    # flag: the shard kernel pushes its keys itself and the merges wait
    # themselves; ll: only the one-launch select exchanges keys, so these
    # stage-by-stage calls (more than 128 rows, the bench's untimed byte
    # count) go through the library all-gather; launch: push + wait launches
    def shard_keys(self, idx_q, layer, plan, q_pos, rp):
        return self.ops.route_shard_keys(
            idx_q, layer["kbar"], block_offset=plan.lo, nblk_local=plan.hi - plan.lo,
            nblk_total=plan.nblk_total, q_pos=q_pos, rows_per_seq=idx_q.shape[0],
            block_table=layer.get("kbar_table"), push=self.keys_x.peer if self.mode == "flag" else None, **rp)

    def gather_keys(self, keys, world):
        if self.mode == "launch":
            return self.keys_x(keys)
        if self.mode == "ll":
            return self.all_gather(keys, world)
        return self.keys_x.slots(keys.shape, keys.dtype)   # filled by the peers' shard kernels

    def merge_keys(self, keys, plan, rp):
        p = {k: v for k, v in rp.items() if k not in ("block_size", "local_blocks")}
        return self.ops.route_merge_keys(keys, nblk_total=plan.nblk_total, own=(plan.lo, plan.hi),
                                         want=("topi32", "bias"),
                                         wait=self.keys_x.peer if self.mode == "flag" else None, **p)

    def select(self, idx_q, layer, plan, q_pos, rp):
        # fused: one launch per layer does the shard keys, the key exchange
        # and the merge (up to 128 rows: each row's merging CTA waits resident)
        if self.fused and plan.world > 1 and idx_q.shape[0] <= 128:
            return self._shard_select(idx_q, layer, plan, q_pos, rp, self.keys_x.peer)
        return super().select(idx_q, layer, plan, q_pos, rp)

    def attend(self, q, layer, topi, bias, q_pos, *, block_size, local_blocks, sm_scale, skip_local,
               out_dtype=torch.float32):
        if not self.fused or out_dtype != torch.float32:
            return super().attend(q, layer, topi, bias, q_pos, block_size=block_size, local_blocks=local_blocks,
                                  sm_scale=sm_scale, skip_local=skip_local, out_dtype=out_dtype)
        # fused: the attend stores its partial into every rank's region
        # itself (no push launch); flag: its local copy must be this rank's
        # own slot, ll: any buffer
        N, H, D = q.shape
        n4 = -(-(N * H * D + N * H) // 4) * 4
        if self.mode == "flag":
            buf = self.part_x.own_slot((n4,), torch.float32)
        else:
            buf = torch.empty(n4, device=q.device, dtype=torch.float32)
        out, lse = buf[:N * H * D].view(N, H, D), buf[N * H * D:N * H * D + N * H].view(N, H)
        return self.ops.decode_attend(q, layer["k_cache"], layer["v_cache"], topi, bias, block_size=block_size,
                                      local_blocks=local_blocks, sm_scale=sm_scale, out=out,
                                      block_table=layer["block_table"], q_pos=q_pos, rows_per_req=N, lse=True,
                                      skip_local=skip_local, lse_out=lse, overlap=True, push=self.part_x.peer)

    def attend_merge(self, q, layer, topi, bias, q_pos, *, block_size, local_blocks, sm_scale, skip_local,
                     out_dtype):
        """ll: the attend also exchanges and merges the partials (one launch
        instead of attend + merge); None when its grid would not be resident
        at once (the caller then attends and merges separately)."""
        if self.mode != "ll":
            return None
        N, H, D = q.shape
        n4 = -(-(N * H * D + N * H) // 4) * 4
        buf = torch.empty(n4, device=q.device, dtype=torch.float32)
        out, lse = buf[:N * H * D].view(N, H, D), buf[N * H * D:N * H * D + N * H].view(N, H)
        final = torch.empty(N, H, D, device=q.device, dtype=out_dtype)
        try:
            return self.ops.decode_attend(q, layer["k_cache"], layer["v_cache"], topi, bias, block_size=block_size,
                                          local_blocks=local_blocks, sm_scale=sm_scale, out=out,
                                          block_table=layer["block_table"], q_pos=q_pos, rows_per_req=N, lse=True,
                                          skip_local=skip_local, lse_out=lse, overlap=True, push=self.part_x.peer,
                                          merged_out=final)
        except NotImplementedError:
            return None

    def exchange_partials(self, o_part, lse_part, world):
        if self.mode == "ll":   # the merge reads the LL words from the region itself
            return o_part, lse_part
        return super().exchange_partials(o_part, lse_part, world)

    def gather_partials(self, buf, world):
        # flag: the attend has already stored the partials into every region
        return self.part_x.slots(buf.shape, buf.dtype) if self.fused else self.part_x(buf)

    def lse_merge(self, o_parts, lse_parts, out_dtype):
        if self.mode == "ll":
            N, H, D = o_parts.shape
            return self.ops.lse_merge_exchange(self.part_x.peer, self.part_x.world, N, H, D, o_parts.device,
                                               out_dtype=out_dtype)[0]
        return self.ops.lse_merge(o_parts, lse_parts, out_dtype=out_dtype,
                                  wait=self.part_x.peer if self.fused else None)[0]

    def check(self):
        self.keys_x.check()
        self.part_x.check()

    def close(self):
        """Collective: every rank calls it once its GPU work is done."""
        import torch.distributed as dist
        torch.cuda.synchronize()
        if dist.is_initialized():
            dist.barrier(group=self.group)
        for x in (self.keys_x, self.part_x):
            x.close_mappings()
        if dist.is_initialized():
            dist.barrier(group=self.group)
        for x in (self.keys_x, self.part_x):
            x.close()


class SplitKVDecode:
    """Decode step of one layer for the rows of one sequence (all rows share
    the sequence; ``q_pos`` holds their global positions)."""

    def __init__(self, *, nblk_total, nblk_filled, block_size, local_blocks, topk, topm, idx_scale, floor,
                 sigma, sm_scale, rank=0, world=1, backend=None):
        self.plan = ShardPlan(nblk_total, world, rank, nblk_filled)
        self.block_size = block_size
        self.local_blocks = local_blocks
        self.sm_scale = sm_scale
        self.rp = dict(block_size=block_size, local_blocks=local_blocks, topk=topk, topm=topm,
                       idx_scale=idx_scale, floor=floor, sigma=sigma)
        self.backend = backend if backend is not None else CudaBackend()

    def window_owner(self, p_max: int, p_min: int) -> int:
        """Rank owning the window of rows at positions [p_min, p_max]; the
        window must not straddle two ranks."""
        lw = self.local_blocks * self.block_size
        first = max(p_min - lw + 1, 0) // self.block_size
        last = p_max // self.block_size
        own = self.plan.owner(last)
        if self.plan.owner(first) != own:
            raise ValueError("the local window spans two shards: give the last shard at least "
                             "local_blocks + 1 blocks before the current one")
        return own

    def step(self, q, idx_q, q_pos, layer, p_range, out_dtype=torch.bfloat16):
        """q [N,H,D], idx_q [N,d], q_pos [N] int64 (device), layer: this
        rank's {kbar, k_cache, v_cache, block_table (global block ids, [1, W]),
        optional kbar_table}.  p_range = (min, max) of q_pos, known on the
        host (a decode loop knows its positions; reading them back from the
        device would stall every layer).  Returns o [N,H,D] (out_dtype)."""
        be, plan, world = self.backend, self.plan, self.plan.world
        if p_range is None:
            raise ValueError("SplitKVDecode.step needs p_range = (min, max) of q_pos on the host")
        # host-only check first: a bad plan fails before any launch or collective
        owner = self.window_owner(int(p_range[1]), int(p_range[0]))
        select = getattr(be, "select", None)                                 # steps 1-3
        if select is not None:
            sel = select(idx_q, layer, plan, q_pos, self.rp)
        else:
            keys = be.shard_keys(idx_q, layer, plan, q_pos, self.rp)        # [N, M]
            sel = be.merge_keys(be.gather_keys(keys, world), plan, self.rp)  # [world, N, M] -> selection
        kw = dict(block_size=self.block_size, local_blocks=self.local_blocks, sm_scale=self.sm_scale,
                  skip_local=(plan.rank != owner))
        attend_merge = getattr(be, "attend_merge", None)      # steps 4-5 in one launch
        if world > 1 and attend_merge is not None:
            out = attend_merge(q, layer, sel["topi32_own"], sel["bias"], q_pos, out_dtype=out_dtype, **kw)
            if out is not None:
                return out
        # one rank: its output is final, written in out_dtype; else fp32 partials
        o_part, lse_part = be.attend(q, layer, sel["topi32_own"], sel["bias"], q_pos,
                                     block_size=self.block_size, local_blocks=self.local_blocks,
                                     sm_scale=self.sm_scale, skip_local=(plan.rank != owner),
                                     out_dtype=out_dtype if world == 1 else torch.float32)
        if world == 1:
            return o_part
        o_all, lse_all = be.exchange_partials(o_part, lse_part, world)      # [world,N,H,D], [world,N,H]
        return be.lse_merge(o_all, lse_all, out_dtype)
