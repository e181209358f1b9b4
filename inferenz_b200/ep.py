"""Expert parallelism for the MoE layer: experts sharded over ranks, tokens over ranks, two all-to-all exchanges.

Rank g of G owns experts [g*E/G, (g+1)*E/G) and its share of the batch's tokens. One layer call on every rank:

1. route its tokens (router, softmax, top-k: bit-exact per token, src/model_fwd.c:997-1011);
2. dispatch: send each token's fp32 row once to every rank owning at least one of its selected experts, with the
   token's (local expert index or -1, weight) for that rank -- all-to-all;
3. run the experts it owns on the rows it received (libinzg ``inzg_moe_experts``): every expert receives every
   token of the batch that selected it, so its numeric path (decode when it has < 12 tokens or the batch has
   <= 8 tokens, src/model_fwd.c:229-249) and its outputs equal the single-GPU call bit for bit;
4. combine: send each (token, rank-k) output back to the token's rank -- all-to-all -- which adds the ten slots in
   rank order (src/model_fwd.c:1134-1140), again bit for bit.

The exchanges use ``torch.distributed`` (NCCL over NVLink between GPUs; gloo in the CPU tests of this module's
logic). The per-rank compute is a backend: :class:`DeviceBackend` drives libinzg on the rank's GPU.
"""
import torch
import torch.distributed as dist

CUDA_STREAM_LEGACY = 1  # cudaStreamLegacy


def stream_handle(s):
    """The CUDA stream handle libinzg should order a call on for torch stream ``s``: torch's default stream has handle
    0, which libinzg reads as "the context's own stream", so it is passed as cudaStreamLegacy (what handle 0 means to
    CUDA) to keep the call ordered with torch's work on that stream."""
    return s.cuda_stream or CUDA_STREAM_LEGACY


class DeviceBackend:
    """libinzg on this rank's GPU: a MoePool holding experts [e_first, e_first + n_local) of every layer used."""

    def __init__(self, pool, stream=None):
        self.pool = pool
        self.stream = stream

    def _st(self):
        s = self.stream if self.stream is not None else torch.cuda.current_stream(self.pool.device)
        return stream_handle(s)

    def route(self, layer, x, bias=None):
        n = x.shape[0]
        sel = torch.empty((n, self.pool.topk), dtype=torch.int32, device=x.device)
        w = torch.empty((n, self.pool.topk), dtype=torch.float32, device=x.device)
        self.pool.route_device(layer, n, x.data_ptr(), sel.data_ptr(), w.data_ptr(),
                               None if bias is None else bias.data_ptr(), self._st())
        return sel, w

    def experts(self, layer, x, sel, w, n_batch):
        m = x.shape[0]
        out = torch.empty((m, self.pool.topk, self.pool.hidden), dtype=torch.float32, device=x.device)
        if m:
            self.pool.experts_device(layer, m, x.data_ptr(), sel.data_ptr(), w.data_ptr(), n_batch, out.data_ptr(),
                                     self._st())
        return out

    def combine(self, slots):
        n = slots.shape[0]
        y = torch.empty((n, slots.shape[2]), dtype=torch.float32, device=slots.device)
        self.pool.combine_device(n, slots.data_ptr(), y.data_ptr(), self._st())
        return y

    def shared(self, layer, x, y, n_batch):
        """y += sigmoid(gate . x) * shared_expert(x) in place (the pool's shared expert of `layer`)."""
        if x.shape[0]:
            self.pool.shared_device(layer, x.shape[0], x.data_ptr(), y.data_ptr(), n_batch, self._st())
        return y


class ExpertParallelMoE:
    """The routed MoE layer over ``world`` ranks with ``n_expert / world`` experts each (see the module docstring)."""

    def __init__(self, backend, n_expert, topk, hidden, rank=None, world=None, group=None, shared_layers=()):
        self.be = backend
        self.shared_layers = set(shared_layers)  # layers whose shared expert (replicated) each rank applies
        self.E, self.K, self.H = n_expert, topk, hidden
        self.group = group
        self.rank = dist.get_rank(group) if rank is None else rank
        self.world = dist.get_world_size(group) if world is None else world
        if n_expert % self.world:
            raise ValueError("n_expert must be a multiple of the number of ranks")
        self.e_per = n_expert // self.world
        self.last = {}

    def expert_range(self, rank=None):
        r = self.rank if rank is None else rank
        return r * self.e_per, self.e_per

    def _a2a(self, out, inp, out_splits, in_splits):
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def moe_block(self, layer, x, bias=None, n_batch=None, stats=False):
        """y [n][H] for this rank's tokens x [n][H] (fp32, on the backend's device). stats: also count the local
        experts that received tokens (self.last["local_units"]; one extra device synchronisation)."""
        G, K, H = self.world, self.K, self.H
        dev = x.device
        n = x.shape[0]
        if n_batch is None:
            t = torch.tensor([n], dtype=torch.int64, device=dev)
            dist.all_reduce(t, group=self.group)
            n_batch = int(t.item())
        sel, w = self.be.route(layer, x, bias)
        owner = (sel // self.e_per).long()                                   # [n][K] rank owning each selection
        hit = torch.zeros((n, G), dtype=torch.bool, device=dev)
        hit.scatter_(1, owner, True)                                         # token t goes to rank d once
        pairs = hit.t().nonzero()                                            # (d, t), d-major, t ascending
        send_d, send_t = pairs[:, 0], pairs[:, 1]
        send_counts = hit.sum(0).to(torch.int64)
        recv_counts = torch.empty_like(send_counts)
        self._a2a(recv_counts, send_counts, None, None)
        sel_t, own_t = sel[send_t], owner[send_t]
        local = torch.where(own_t == send_d[:, None], sel_t - (send_d[:, None] * self.e_per).to(torch.int32),
                            torch.full_like(sel_t, -1))
        meta_send = torch.cat([local, w[send_t].view(torch.int32)], 1).contiguous()
        x_send = x[send_t].contiguous()
        s_splits, r_splits = send_counts.tolist(), recv_counts.tolist()
        m = sum(r_splits)
        x_recv = torch.empty((m, H), dtype=torch.float32, device=dev)
        meta_recv = torch.empty((m, 2 * K), dtype=torch.int32, device=dev)
        self._a2a(x_recv, x_send, r_splits, s_splits)
        self._a2a(meta_recv, meta_send, r_splits, s_splits)
        sel_recv = meta_recv[:, :K].contiguous()
        w_recv = meta_recv[:, K:].contiguous().view(torch.float32)
        out = self.be.experts(layer, x_recv, sel_recv, w_recv, n_batch)     # [m][K][H]
        present = sel_recv >= 0
        back = out[present].contiguous()                                     # (row, k) row-major
        rows_src = torch.repeat_interleave(torch.arange(G, device=dev), torch.tensor(r_splits, device=dev))
        back_counts = torch.zeros(G, dtype=torch.int64, device=dev)
        back_counts.index_add_(0, rows_src, present.sum(1).to(torch.int64))
        home_counts = torch.bincount(owner.flatten(), minlength=G).to(torch.int64)
        b_send, b_recv = back_counts.tolist(), home_counts.tolist()
        res = torch.empty((sum(b_recv), H), dtype=torch.float32, device=dev)
        self._a2a(res, back, b_recv, b_send)
        # results arrive per owner rank d; inside d in this rank's send order (t ascending, then k ascending)
        tk = torch.cat([(owner == d).nonzero() for d in range(G)], 0)
        slots = torch.empty((n, K, H), dtype=torch.float32, device=dev)
        slots[tk[:, 0], tk[:, 1]] = res
        self.last = {"sel": sel, "w": w, "m": m, "dispatch_rows": int(x_send.shape[0]), "results": int(res.shape[0])}
        y = self.be.combine(slots)
        if layer in self.shared_layers:
            y = self.be.shared(layer, x, y, n_batch)
        if stats:
            used = sel_recv[present].long()
            self.last["local_units"] = int((torch.bincount(used, minlength=self.e_per) > 0).sum()) if used.numel() else 0
        return y

    def moe_block_fixed(self, layer, x, bias=None, n_batch=None, capacity=None):
        """The same layer with fixed-size exchanges: every rank sends each rank a block of ``capacity`` token rows
        (its n <= capacity tokens, entries of other ranks marked -1) and receives a block of ``capacity`` x topk
        results back, so no count crosses to the host and the step can be captured in a CUDA graph. For decode-sized
        batches; the bytes grow with world x capacity x topk."""
        G, K, H = self.world, self.K, self.H
        dev = x.device
        n = x.shape[0]
        C = n if capacity is None else capacity
        if n > C:
            raise ValueError("more tokens than the exchange capacity")
        nb = n_batch if n_batch is not None else n * G
        sel, w = self.be.route(layer, x, bias)
        owner = (sel // self.e_per).to(torch.int32)                          # [n][K]
        d = torch.arange(G, device=dev, dtype=torch.int32)[:, None, None]     # [G][1][1]
        local = torch.where(owner[None] == d, sel[None] - d * self.e_per, torch.full_like(sel[None], -1))  # [G][n][K]
        meta_send = torch.full((G, C, 2 * K), -1, dtype=torch.int32, device=dev)
        meta_send[:, :n, :K] = local
        meta_send[:, :n, K:] = w.view(torch.int32)[None]
        x_send = torch.zeros((G, C, H), dtype=torch.float32, device=dev)
        x_send[:, :n] = x[None]
        x_recv = torch.empty_like(x_send)
        meta_recv = torch.empty_like(meta_send)
        self._a2a(x_recv, x_send, None, None)
        self._a2a(meta_recv, meta_send, None, None)
        meta_recv = meta_recv.view(G * C, 2 * K)
        out = self.be.experts(layer, x_recv.view(G * C, H), meta_recv[:, :K].contiguous(),
                              meta_recv[:, K:].contiguous().view(torch.float32), nb)  # [G*C][K][H]
        back = torch.empty_like(out)
        self._a2a(back, out, None, None)                                     # block d: rank d's results for my rows
        idx = (owner.long() * C + torch.arange(n, device=dev)[:, None]) * K + torch.arange(K, device=dev)[None, :]
        slots = back.view(G * C * K, H)[idx.view(-1)].view(n, K, H)
        y = self.be.combine(slots)
        if layer in self.shared_layers:
            y = self.be.shared(layer, x, y, nb)
        return y


class PeerExchangeMoE:
    """The expert-parallel layer with the exchange inside libinzg (``inzg_ep_*``): each rank's pool holds its
    ``n_expert / world`` experts; every (token, owning rank) row and every owned output slot crosses NVLink once,
    written by the library's kernels straight into the peer's memory, with device-side epoch flags instead of host
    synchronisation or a collective. The step (route, dispatch, owned experts, return, rank-order combine, shared
    expert) runs as one CUDA graph per shape; outputs equal the single-GPU call bit for bit.

    The handles are exchanged once over ``group`` (any backend: ``all_gather_object``)."""

    def __init__(self, pool, capacity, group=None, rank=None, world=None):
        self.pool = pool
        self.group = group
        self.rank = dist.get_rank(group) if rank is None else rank
        self.world = dist.get_world_size(group) if world is None else world
        self.capacity = capacity
        handle = pool.ep_attach(self.rank, self.world, capacity)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=group)
        pool.ep_connect(handles)

    def moe_block(self, layer, x, bias=None, n_batch=None, y=None, stream=None):
        """y [n][H] for this rank's n <= capacity tokens x [n][H] (fp32, on the pool's device). n_batch: the whole
        batch's token count (default: n on every rank)."""
        n = x.shape[0]
        if y is None:
            y = torch.empty_like(x)
        s = stream if stream is not None else torch.cuda.current_stream(x.device)
        self.pool.ep_forward_device(layer, n, x.data_ptr(), y.data_ptr(), n * self.world if n_batch is None else n_batch,
                                    None if bias is None else bias.data_ptr(), stream_handle(s))
        return y

    def barrier(self, stream=None):
        """Device-side rendezvous of all ranks on ``stream`` (outside any step)."""
        s = stream if stream is not None else torch.cuda.current_stream(self.pool.device)
        self.pool.ep_barrier(stream_handle(s))

    def close(self):
        self.pool.ep_detach()


__all__ = ["DeviceBackend", "ExpertParallelMoE", "PeerExchangeMoE", "stream_handle"]
