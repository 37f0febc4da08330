"""Expert parallelism of the MoE block across the GPUs of one node.

GPU g of N owns experts [g*E/N, (g+1)*E/N) of every layer and holds the whole
router.  For its own tokens each GPU
  1. routes them (rmsnorm + exact router + top-k: rbt_moe_route_device),
  2. plans the dispatch: a token goes to every GPU that owns at least one of its
     top-k experts, once per GPU (rbt_ep_plan),
  3. exchanges the per-GPU row counts, then the token rows together with their
     expert ids (local to the receiving GPU, -1 for slots computed elsewhere) and
     combine weights, as one [rows, D + 2K] f32 all-to-all (the ids travel as
     their bit patterns; rbt_ep_pack builds the send buffers),
  4. runs its experts on the rows it received: one partial output row per row,
     the weighted sum over its own slots in selection order
     (rbt_moe_experts_device),
  5. returns the partial rows (NCCL all-to-all), and adds them to the residual in
     ascending GPU order (rbt_ep_combine).
This is the expert-parallel form of rabbit2.c:512-542; the routing is bit-exact
and the outputs differ from the one-GPU call only by the order of the final fp32
additions.  The collectives are torch.distributed calls on whatever process group
the caller initialised (NCCL on GPUs); the arithmetic is librbt_moe's.

`ops` carries the per-GPU steps.  GpuOps is the product (librbt_moe kernels on
the rank's GPU); the CPU tests substitute host implementations of the same five
steps to check the exchange logic with the gloo backend.
"""
import torch
import torch.distributed as dist

from . import moe


class GpuOps:
    """The five per-GPU steps on librbt_moe (device tensors of this rank's GPU)."""

    def __init__(self, ctx: moe.MoeContext, n_ranks: int):
        self.ctx, self.lib = ctx, ctx.lib
        self.D, self.E, self.K = ctx.D, ctx.E, ctx.K
        self.n_ranks = n_ranks
        self.epr = self.E // n_ranks
        self.device = torch.device("cuda", torch.cuda.current_device())

    def _stream(self):
        return torch.cuda.current_stream().cuda_stream

    def _check(self, ok):
        if not ok:
            raise moe.RbtMoeError(self.lib.rbt_moe_last_error().decode())

    def route(self, layer, x, xb, idx, wt, block):
        self.ctx.route_device(layer, x, xb, idx, wt, block=block, stream=self._stream())

    def plan(self, idx, pos, counts, capacity=0):
        self._check(self.lib.rbt_ep_plan(idx.data_ptr(), idx.shape[0], self.K, self.n_ranks, self.epr, capacity,
                                         pos.data_ptr(), counts.data_ptr(), self._stream()))

    def pack(self, xb, idx, wt, pos, counts, send_rows, send_idx, send_wt):
        self._check(self.lib.rbt_ep_pack(xb.data_ptr(), idx.data_ptr(), wt.data_ptr(), xb.shape[0], self.D, self.K,
                                         self.n_ranks, self.epr, pos.data_ptr(), counts.data_ptr(),
                                         send_rows.data_ptr(), send_idx.data_ptr(), send_wt.data_ptr(),
                                         self._stream()))

    def experts(self, layer, rows, idx, wt, out):
        self.ctx.experts_device(layer, rows, idx, wt, out, stream=self._stream())

    def combine(self, x, pos, counts, back, out):
        self._check(self.lib.rbt_ep_combine(x.data_ptr() if x is not None else None, out.shape[0], self.D,
                                            self.n_ranks, pos.data_ptr(), counts.data_ptr(),
                                            back.data_ptr() if back.numel() else None, out.data_ptr(),
                                            self._stream()))


class ExpertParallelMoe:
    """The MoE block of every layer, expert-parallel over a process group.

    capacity: with every rank calling with at most `capacity` tokens, each rank
    sends a fixed segment of `capacity` rows to every GPU (rows not routed there
    carry no slots), so no row count has to reach the host: no synchronisation,
    and the whole call can be captured in a CUDA graph.  Meant for decode-sized
    calls; without it the exact counts are exchanged first (one host read per call).
    """

    def __init__(self, ops, group=None, capacity=None):
        self.ops, self.group, self.capacity = ops, group, capacity
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if ops.E % self.world:
            raise ValueError(f"{ops.E} experts do not split evenly over {self.world} GPUs")
        self.last_counts = None  # (rows sent to each GPU, rows received from each GPU) of the last call

    def _a2a(self, out, inp, out_splits, in_splits):
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def forward(self, layer, x, block=True, out=None):
        """block: x += MoE(rmsnorm(x)) in place and returns x; otherwise returns MoE(x) (in `out` if given)."""
        o = self.ops
        T, D, K, R = x.shape[0], o.D, o.K, self.world
        dev = x.device
        xb = torch.empty_like(x)
        idx = torch.empty((T, K), dtype=torch.int32, device=dev)
        wt = torch.empty((T, K), dtype=torch.float32, device=dev)
        pos = torch.empty((T, R), dtype=torch.int32, device=dev)
        counts = torch.zeros(R, dtype=torch.int32, device=dev)
        cap = self.capacity if self.capacity and T <= self.capacity else 0
        if T:
            o.route(layer, x, xb, idx, wt, block)
            o.plan(idx, pos, counts, cap) if cap else o.plan(idx, pos, counts)
        if cap:
            send_splits = recv_splits = [cap] * R
        else:
            recv_counts = torch.empty(R, dtype=torch.int32, device=dev)
            self._a2a(recv_counts, counts, [1] * R, [1] * R)
            both = torch.stack([counts, recv_counts]).cpu()  # the one host synchronisation of the call
            send_splits, recv_splits = both[0].tolist(), both[1].tolist()
        self.last_counts = (send_splits, recv_splits)
        n_send, n_recv = sum(send_splits), sum(recv_splits)
        send_rows = torch.empty((n_send, D), dtype=torch.float32, device=dev)
        send_idx = torch.empty((n_send, K), dtype=torch.int32, device=dev)
        if cap:
            send_idx.fill_(-1)
        send_wt = torch.empty((n_send, K), dtype=torch.float32, device=dev)
        if T:
            o.pack(xb, idx, wt, pos, counts, send_rows, send_idx, send_wt)
        # one exchange for a row, its expert ids (their bits carried as f32) and its weights
        send = torch.cat([send_rows, send_idx.view(torch.float32), send_wt], dim=1)
        recv = torch.empty((n_recv, D + 2 * K), dtype=torch.float32, device=dev)
        self._a2a(recv, send, recv_splits, send_splits)
        recv_rows = recv[:, :D].contiguous()
        recv_idx = recv[:, D:D + K].contiguous().view(torch.int32)
        recv_wt = recv[:, D + K:].contiguous()
        partial = torch.empty((n_recv, D), dtype=torch.float32, device=dev)
        if n_recv:
            o.experts(layer, recv_rows, recv_idx, recv_wt, partial)
        back = torch.empty((n_send, D), dtype=torch.float32, device=dev)
        self._a2a(back, partial, send_splits, recv_splits)
        if block:
            if T:
                o.combine(x, pos, counts, back, x)
            return x
        res = out if out is not None else torch.empty_like(x)
        if T:
            o.combine(None, pos, counts, back, res)
        return res

    def block(self, layer, x):
        return self.forward(layer, x, block=True)

    def ffn(self, layer, xb, out=None):
        return self.forward(layer, xb, block=False, out=out)
