"""Ulysses-style sequence <-> head re-sharding around the BSA call (one process per GPU).

The DiT runs sequence-sharded ([B, H, S/P, D] per rank); BSA needs whole sequences because a
query block may select any KV block.  Heads are independent, so one all-to-all turns the
sequence shard of all heads into all tokens of H/P heads, BSA runs locally on those heads, and a
second all-to-all returns the output to sequence shards.  The upstream PyTorch model did this
with ``ulysses_wrapper`` / ``context_parallel_util``, which the MLX port dropped
(rope_3d.py:14; stubbed in tests/parity/test_dit_block_parity.py:88-112).

Two exchanges move the pieces (``ulysses_bsa_attention``): on CUDA tensors of an NCCL group the
default is ``PeerExchange`` -- persistent CUDA-IPC buffers and copies on the copy engines over NVLink,
ordered by three 4-byte NCCL all-reduces per call -- and otherwise point-to-point messages of the
process group (NCCL, or gloo on CPU for tests).  ``seq_to_heads`` / ``heads_to_seq`` are the plain
``all_to_all_single`` forms.  Pre-RoPE Q/K travel and RoPE is applied after the exchange, because the
rotation needs each token's global position.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.distributed as dist

from .models.block_sparse_attention import bsa_attention

__all__ = ["seq_to_heads", "heads_to_seq", "ulysses_bsa_attention", "PeerExchange", "close_exchanges",
           "exchange_copy_plan"]


def _world(group) -> int:
    return dist.get_world_size(group) if dist.is_initialized() else 1


def seq_to_heads(x: torch.Tensor, group=None) -> torch.Tensor:
    """[..., B, H, S/P, D] sequence shard (rank r holds tokens r*S/P .. (r+1)*S/P - 1 of every
    head) -> [..., B, H/P, S, D] head shard (rank r holds heads r*H/P .. (r+1)*H/P - 1)."""
    P = _world(group)
    if P == 1:
        return x
    *lead, B, H, Sl, D = x.shape
    if H % P:
        raise ValueError(f"{H} heads do not split over {P} ranks")
    L = len(lead)
    y = x.reshape(*lead, B, P, H // P, Sl, D)
    # bring the destination-rank axis to the front: [P, lead..., B, H/P, Sl, D]
    y = y.movedim(L + 1, 0).contiguous()
    recv = torch.empty_like(y)
    dist.all_to_all_single(recv, y, group=group)
    # recv[p] = rank p's sequence shard of my heads -> concatenate along the sequence axis
    recv = recv.movedim(0, L + 2)  # [lead..., B, H/P, P, Sl, D]
    return recv.reshape(*lead, B, H // P, P * Sl, D)


def heads_to_seq(o: torch.Tensor, group=None) -> torch.Tensor:
    """Inverse of ``seq_to_heads``: [..., B, H/P, S, D] -> [..., B, H, S/P, D]."""
    P = _world(group)
    if P == 1:
        return o
    *lead, B, Hl, S, D = o.shape
    if S % P:
        raise ValueError(f"S={S} does not split over {P} ranks")
    L = len(lead)
    y = o.reshape(*lead, B, Hl, P, S // P, D)
    y = y.movedim(L + 2, 0).contiguous()  # [P, lead..., B, Hl, Sl, D]
    recv = torch.empty_like(y)
    dist.all_to_all_single(recv, y, group=group)
    recv = recv.movedim(0, L + 1)  # [lead..., B, P, Hl, Sl, D]
    return recv.reshape(*lead, B, P * Hl, S // P, D)


def _exchange_in(q, k, v, heads, P: int, rank: int, group):
    """Post the exchange that gives this rank whole sequences of its heads of one head group.

    heads: the group's global head ids; rank p owns heads[p*Hl:(p+1)*Hl].  Every [S/P, D] piece
    moves as its own point-to-point message straight from the input shard into the
    whole-sequence buffer [3, B, Hl, S, D], so no packing copy runs on either side.  Peers post
    their messages in the same (tensor, batch, head) order, which pairs sends with receives.
    Returns (works, qkv_h).
    """
    B, _, Sl, D = q.shape
    Hl = len(heads) // P
    qkv_h = torch.empty((3, B, Hl, P * Sl, D), device=q.device, dtype=q.dtype)
    ops = []
    for t, x in enumerate((q, k, v)):
        for b in range(B):
            for p in range(P):
                for j in range(Hl):
                    if p == rank:
                        qkv_h[t, b, j, rank * Sl:(rank + 1) * Sl].copy_(x[b, heads[rank * Hl + j]])
                    else:
                        ops.append(dist.P2POp(dist.isend, x[b, heads[p * Hl + j]], p, group))
                        ops.append(dist.P2POp(dist.irecv, qkv_h[t, b, j, p * Sl:(p + 1) * Sl], p, group))
    works = dist.batch_isend_irecv(ops) if ops else []
    return works, qkv_h


def _exchange_out(o, out, heads, P: int, rank: int, group):
    """Inverse of ``_exchange_in`` for the output: o [B, Hl, S, D] (this rank's heads, whole
    sequence) -> out[:, heads] [B, H, S/P, D] (every head of the group, this rank's tokens)."""
    B, Hl, S, D = o.shape
    Sl = S // P
    ops = []
    for b in range(B):
        for p in range(P):
            for j in range(Hl):
                if p == rank:
                    out[b, heads[rank * Hl + j]].copy_(o[b, j, rank * Sl:(rank + 1) * Sl])
                else:
                    ops.append(dist.P2POp(dist.isend, o[b, j, p * Sl:(p + 1) * Sl], p, group))
                    ops.append(dist.P2POp(dist.irecv, out[b, heads[p * Hl + j]], p, group))
    return dist.batch_isend_irecv(ops) if ops else []


def _head_groups(H: int, P: int, groups: Optional[int]) -> int:
    """Head groups of the pipelined exchange: more groups hide more of the first pull and the last push but
    add per-group launch latency and attention tails.  Measured at config 2 (32 heads): 2 GPUs 6.66 / 6.80 /
    7.11 ms per call with 2 / 4 / 8 groups; 8 GPUs 2.60 / 2.56 ms with 2 / 4."""
    if groups is None:
        groups = min(2 if P <= 4 else 4, H // P) if H >= P else 1
    groups = max(1, int(groups))
    while groups > 1 and (H % groups or (H // groups) % P):
        groups -= 1
    return groups


# SMs left to the message exchange's kernels while the persistent attention kernel runs
DEFAULT_SM_RESERVE = 8


# copy streams per direction (peers are spread over them: two copy engines share a group's pull; 2.34
# against 2.56 ms per config-2 call at 8 GPUs) and compute streams (groups alternate)
COPY_STREAMS = 2
COMPUTE_STREAMS = 2


def exchange_copy_plan(P: int, r: int, B: int, H: int, Sl: int, D: int, elt: int, G: int, stage, outr, recv_in,
                       o_slot, nin: int = 1, nout: int = 1):
    """The copies of one ``PeerExchange`` call on rank r, as bsa_copy_3d rows (dst, dpitch, dslice, src, spitch,
    sslice, width, height, depth) in bytes.  stage[p] / outr[p]: rank p's stage [3, B, H, S/P, D] and
    out_recv [B, H, S/P, D] (mapped here); recv_in[slot] [3, B, Hl, S, D] and o_slot[slot] [B, Hl, S, D]: this
    rank's two input and output slots.  Returns (pull, push): per head group, per copy stream, a list of rows.

    The copy engine pays a fixed cost per call, so a pull moves q, k and v of the group's heads from one peer
    in one 3-D copy (slices: the tensors; rows: the heads; a row: the peer's token range of one head)."""
    S, Hg = Sl * P, H // G
    Hl = Hg // P
    piece, row = Sl * D * elt, S * D * elt
    pull, push = [], []
    for g in range(G):
        sl = g % 2
        h0 = g * Hg + r * Hl  # first head of this group that rank r computes
        ins = [[] for _ in range(nin)]
        for p in range(P):
            for b in range(B):
                src = stage[p] + (b * H + h0) * piece
                dst = recv_in[sl] + (b * Hl * S + p * Sl) * D * elt
                ins[(p + r) % nin].append((dst, row, B * Hl * row, src, piece, B * H * piece, piece, Hl, 3))
        outs = [[] for _ in range(nout)]
        for p in range(P):
            for b in range(B):
                src = o_slot[sl] + (b * Hl * S + p * Sl) * D * elt
                dst = outr[p] + (b * H + h0) * piece
                outs[(p + r) % nout].append((dst, piece, piece * Hl, src, row, row * Hl, piece, Hl, 1))
        pull.append(ins)
        push.append(outs)
    return pull, push


class PeerExchange:
    """Copy-engine all-to-all for the sequence-parallel BSA call (one per process group and shape).

    Persistent buffers, mapped by every rank of the node once (CUDA IPC):
      stage    [3, B, H, S/P, D]  this rank's q/k/v shard, which peers read
      out_recv [B, H, S/P, D]     this rank's output shard, which peers write
    and local ones: two whole-sequence input slots [3, B, Hl, S, D] and two output slots
    [B, Hl, S, D] (Hl = heads of one group owned by this rank).

    One call: stage group 0's heads of q/k/v (local copy), barrier, stage the other groups, barrier;
    per head group g a copy-in stream pulls the group's q/k/v pieces from every peer's stage into slot
    g%2 (one 3-D copy per peer and batch; group 0 right after the first barrier, the others after the
    second), the compute stream runs BSA on it, and a copy-out stream pushes each peer's token range of
    the output straight into that peer's out_recv.  A final barrier (after this rank's last push) means
    every peer's pushes into this rank's out_recv are complete.  Copy engines carry every transfer
    over NVLink, so the attention kernel keeps all SMs.  Three barriers per call (two with one head
    group; a 4-byte all-reduce each); no host synchronisation.  The copy plan of every group is built
    once (``_plan``) and issued with one host call per stream.
    """

    def __init__(self, B: int, H: int, Sl: int, D: int, dtype: torch.dtype, groups: int, group, device):
        from . import _native

        self.P = _world(group)
        self.rank = dist.get_rank(group)
        self.group = group
        self.device = device
        self.B, self.H, self.Sl, self.D, self.dtype, self.G = B, H, Sl, D, dtype, groups
        self.Hg = H // groups
        self.Hl = self.Hg // self.P
        self.S = Sl * self.P
        self.elt = torch.empty((), dtype=dtype).element_size()
        with torch.cuda.device(device):
            stage_ptr, h_stage = _native.ipc_alloc(3 * B * H * Sl * D * self.elt)
            outr_ptr, h_outr = _native.ipc_alloc(B * H * Sl * D * self.elt)
        self._own = [stage_ptr, outr_ptr]
        handles = [None] * self.P
        dist.all_gather_object(handles, (h_stage, h_outr), group=group)
        self._opened = []
        self.peer_stage, self.peer_outr = [], []
        with torch.cuda.device(device):
            for p in range(self.P):
                if p == self.rank:
                    self.peer_stage.append(stage_ptr)
                    self.peer_outr.append(outr_ptr)
                else:
                    a, b = _native.ipc_open(handles[p][0]), _native.ipc_open(handles[p][1])
                    self._opened += [a, b]
                    self.peer_stage.append(a)
                    self.peer_outr.append(b)
        self.stage = _native.wrap_device(stage_ptr, (3, B, H, Sl, D), dtype, device)
        self.out_recv = _native.wrap_device(outr_ptr, (B, H, Sl, D), dtype, device)
        self.recv_in = [torch.empty((3, B, self.Hl, self.S, D), device=device, dtype=dtype) for _ in range(2)]
        self.o_slot = [torch.empty((B, self.Hl, self.S, D), device=device, dtype=dtype) for _ in range(2)]
        self.flag = torch.zeros((1,), device=device, dtype=torch.int32)
        ncopy = max(1, min(COPY_STREAMS, self.P))
        self.s_in = [torch.cuda.Stream(device) for _ in range(ncopy)]
        self.s_out = [torch.cuda.Stream(device) for _ in range(ncopy)]
        self.s_comp = [torch.cuda.Stream(device) for _ in range(COMPUTE_STREAMS)]
        self.s_join = [torch.cuda.Stream(device) for _ in range(2)]
        self._native = _native
        self._plan()
        # events reused by every call (recording again replaces the previous record; waits already
        # queued keep the record they saw)
        G = self.G
        self.ev_start = torch.cuda.Event()
        self.ev_staged = torch.cuda.Event()
        self.ev_in = [[torch.cuda.Event() for _ in self.s_in] for _ in range(G)]
        self.ev_comp = [torch.cuda.Event() for _ in range(G)]
        self.ev_out = [[torch.cuda.Event() for _ in self.s_out] for _ in range(G)]
        self.ev_push = [torch.cuda.Event() for _ in range(G)]
        self._slot_bufs = {}

    def _plan(self):
        """Every copy of a call, fixed once (``exchange_copy_plan``), packed for one host call per stream."""
        import ctypes

        def pack(rows):
            arr = (ctypes.c_int64 * (9 * max(1, len(rows))))(*[x for rw in rows for x in rw])
            return arr, len(rows)

        pull, push = exchange_copy_plan(self.P, self.rank, self.B, self.H, self.Sl, self.D, self.elt, self.G,
                                        self.peer_stage, self.peer_outr, [t.data_ptr() for t in self.recv_in],
                                        [t.data_ptr() for t in self.o_slot], len(self.s_in), len(self.s_out))
        self.pull = [[pack(x) for x in g] for g in pull]
        self.push = [[pack(x) for x in g] for g in push]

    def slot_buffers(self, sl: int, nb: int, topk: int, scratch_bytes: int):
        """Per-slot routing output and scratch of the compute step (allocated once per size)."""
        key = (sl, nb, topk, scratch_bytes)
        bufs = self._slot_bufs.get(key)
        if bufs is None:
            idx = torch.empty((self.B, self.Hl, nb, topk), device=self.device, dtype=torch.int32)
            scratch = torch.empty((max(16, scratch_bytes),), device=self.device, dtype=torch.uint8)
            bufs = self._slot_bufs[key] = (idx, scratch)
        return bufs

    def _barrier(self):
        dist.all_reduce(self.flag, group=self.group)  # on the current stream; no host wait

    def run(self, q, k, v, compute) -> torch.Tensor:
        """q, k, v: [B, H, S/P, D] shards; compute(qh, kh, vh, out, slot) runs BSA on one group's
        whole-sequence heads [B, Hl, S, D] into out.  Returns the output shard [B, H, S/P, D]."""
        nat = self._native
        C = torch.cuda.current_stream(self.device)
        # stage group 0's heads first: its pulls start while the other groups stage
        hg = self.Hg
        for t, x in enumerate((q, k, v)):
            self.stage[t][:, :hg].copy_(x[:, :hg])
        self._barrier()  # every rank has staged group 0 and finished its previous call
        self.ev_start.record(C)
        for st in self.s_in + self.s_out + self.s_comp:
            st.wait_event(self.ev_start)
        if self.G > 1:
            for t, x in enumerate((q, k, v)):
                self.stage[t][:, hg:].copy_(x[:, hg:])
            self._barrier()  # every rank has staged every group
            self.ev_staged.record(C)
        for g in range(self.G):
            sl = g % 2
            # copy-in: this group's pieces from every peer, one host call per copy stream
            for i, st in enumerate(self.s_in):
                if g == 1:
                    st.wait_event(self.ev_staged)
                if g >= 2:
                    st.wait_event(self.ev_comp[g - 2])  # input slot free
                arr, n = self.pull[g][i]
                nat.copy_3d_list(arr, n, st)
                self.ev_in[g][i].record(st)
            # compute (with COMPUTE_STREAMS > 1 groups alternate between streams, so one group's
            # kernels can start on SMs that the previous group's attention tail leaves idle)
            cs = self.s_comp[g % len(self.s_comp)]
            for ev in self.ev_in[g]:
                cs.wait_event(ev)
            if g >= 2:
                cs.wait_event(self.ev_push[g - 2])  # output slot free
            xin, o = self.recv_in[sl], self.o_slot[sl]
            with torch.cuda.stream(cs):
                compute(xin[0], xin[1], xin[2], o, sl)
            self.ev_comp[g].record(cs)
            # copy-out: each peer's token range of the output straight into its out_recv
            joint = self.s_join[g % 2]
            for i, st in enumerate(self.s_out):
                st.wait_event(self.ev_comp[g])
                arr, n = self.push[g][i]
                nat.copy_3d_list(arr, n, st)
                self.ev_out[g][i].record(st)
                joint.wait_event(self.ev_out[g][i])
            self.ev_push[g].record(joint)
        for st in self.s_in + self.s_out + self.s_comp + self.s_join:
            C.wait_stream(st)
        self._barrier()  # every peer's pushes into this rank's out_recv are complete
        return self.out_recv.clone()

    def close(self):
        """Unmap the peers' buffers, wait until every rank has done the same, free this rank's."""
        torch.cuda.synchronize(self.device)
        for ptr in self._opened:
            self._native.ipc_close(ptr)
        self._opened = []
        dist.barrier(group=self.group)
        torch.cuda.synchronize(self.device)
        for ptr in self._own:
            self._native.ipc_free(ptr)
        self._own = []


_EXCHANGES = {}


def _peer_exchange(q, groups, group) -> Optional[PeerExchange]:
    """The cached copy-engine exchange for this call, or None where it does not apply (CPU
    tensors, a non-NCCL group)."""
    if not q.is_cuda or dist.get_backend(group) != "nccl":
        return None
    B, H, Sl, D = q.shape
    key = (id(group), q.device.index, B, H, Sl, D, q.dtype, groups)
    ex = _EXCHANGES.get(key)
    if ex is None:
        ex = PeerExchange(B, H, Sl, D, q.dtype, groups, group, q.device)
        _EXCHANGES[key] = ex
    return ex


def close_exchanges() -> None:
    """Release the copy-engine exchanges' buffers (call on every rank, before destroy_process_group)."""
    for ex in _EXCHANGES.values():
        ex.close()
    _EXCHANGES.clear()


def ulysses_bsa_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, shape: Tuple[int, int, int],
                          sparsity: float = 0.9375, chunk_thw: Tuple[int, int, int] = (4, 4, 4),
                          sm_scale: Optional[float] = None, *, topk: Optional[int] = None, rope=None,
                          group=None, head_groups: Optional[int] = None,
                          sm_reserve: Optional[int] = None, exchange: str = "auto") -> torch.Tensor:
    """Sequence-sharded BSA: q, k, v are this rank's [B, H, S/P, D] shards; returns the output
    shard [B, H, S/P, D].  ``shape`` is the full latent (T, H, W) of the whole sequence.

    The heads are processed in ``head_groups`` groups (default: 2 up to 4 GPUs, 4 beyond; each a
    multiple of P heads) so the exchanges overlap the compute.  ``exchange``:
      "copy_engine" -- ``PeerExchange``: CUDA IPC buffers and 2-D copies on the copy engines
                       (no SMs taken from the attention kernel); CUDA tensors on an NCCL group;
      "messages"    -- point-to-point messages of the process group (NCCL or gloo) on the
                       communicator's stream, with ``sm_reserve`` SMs kept free of the attention
                       kernel for them;
      "auto"        -- the copy engines where they apply, else messages.
    Every rank posts the same exchanges in the same order.
    """
    P = _world(group)
    if P == 1:
        return bsa_attention(q, k, v, shape, sparsity, chunk_thw, sm_scale, topk=topk, rope=rope)
    if q.shape != k.shape or q.shape != v.shape:
        raise ValueError("q, k, v must have the same shape [B, H, S/P, D]")
    q, k, v = (x.contiguous() for x in (q, k, v))
    B, H, Sl, D = q.shape
    if H % P:
        raise ValueError(f"{H} heads do not split over {P} ranks")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise ValueError("q, k, v must share one dtype")
    rank = dist.get_rank(group)
    G = _head_groups(H, P, head_groups)
    if exchange in ("auto", "copy_engine"):
        ex = _peer_exchange(q, G, group)
        if ex is None and exchange == "copy_engine":
            raise ValueError("the copy-engine exchange needs CUDA tensors and an NCCL process group")
        if ex is not None:
            from . import _native
            from .models.block_sparse_attention import num_selected_blocks

            S = Sl * P
            _native._geometry(S, shape, chunk_thw)
            nb = S // (chunk_thw[0] * chunk_thw[1] * chunk_thw[2])
            k_sel = num_selected_blocks(nb, sparsity) if topk is None else int(topk)
            scale = 1.0 / math.sqrt(D) if sm_scale is None else sm_scale
            rope_arg = rope.native_args() if rope is not None else None
            nbytes = int(_native.lib().bsa_forward_scratch_bytes(B, H // P // G, S, D, *chunk_thw))

            def compute(qh, kh, vh, o, sl):
                idx, scratch = ex.slot_buffers(sl, nb, k_sel, nbytes)
                _native.forward(qh, kh, vh, shape, chunk_thw, k_sel, scale, rope=rope_arg, out=o, block_indices=idx,
                                scratch=scratch)

            return ex.run(q, k, v, compute)
    elif exchange != "messages":
        raise ValueError(f"unknown exchange {exchange!r}")
    reserve = DEFAULT_SM_RESERVE if sm_reserve is None else int(sm_reserve)
    Hg = H // G
    heads = [list(range(g * Hg, (g + 1) * Hg)) for g in range(G)]
    out = torch.empty_like(q)
    pending_in = _exchange_in(q, k, v, heads[0], P, rank, group)
    pending_out = []
    for g in range(G):
        works, qkv_h = pending_in
        # post the next group's exchange before this group's compute so it does not queue behind it
        if g + 1 < G:
            pending_in = _exchange_in(q, k, v, heads[g + 1], P, rank, group)
        for w in works:
            w.wait()
        o = bsa_attention(qkv_h[0], qkv_h[1], qkv_h[2], shape, sparsity, chunk_thw, sm_scale, topk=topk, rope=rope,
                          sm_reserve=reserve if q.is_cuda else 0)
        pending_out.extend(_exchange_out(o, out, heads[g], P, rank, group))
    for w in pending_out:
        w.wait()
    return out
