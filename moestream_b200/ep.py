"""Expert parallelism over the GPUs of one node.

The reference runs one process on one GPU and has no expert parallelism;
this is how the slot-pool MoE layer spreads over n_rank GPUs. Experts are
split evenly and contiguously (expert e lives on rank e // n_local as local
expert e % n_local, all of them resident); tokens are split evenly too, each
rank routing its own tokens. Per layer:

  1. dispatch: each (token, k) row is packed into a fixed-capacity block for
     the rank that owns its expert (bf16 activations with the local expert
     id in the two bf16 columns after them, -1 for unused rows);
  2. one equal-split all-to-all of those rows (no count exchange and no
     host round trip: a destination block holds every row a source can
     send it);
  3. the local FFN over the received rows with top_k = 1 and weight 1
     (unused rows land in the zero slot and give exact zeros);
  4. one equal-split all-to-all of the f32 results back to the source ranks;
  5. combine: y[t] = sum_k w[t, k] * (row of pair (t, k)), k ascending.

The exchange goes through torch.distributed (NCCL on GPUs, gloo on CPU);
dispatch and combine are the library's device kernels, or any functions
with the same meaning passed in (the CPU tests pass the oracle's).
"""
import torch


class ExpertParallel:
    """Buffers and steps of one rank's expert-parallel MoE layer."""

    def __init__(self, world, rank, n_expert, n_tok, top_k, K, device, group=None,
                 dispatch=None, combine=None):
        if n_expert % world or n_tok % world:
            raise ValueError(f"{n_expert} experts and {n_tok} tokens must split evenly over "
                             f"{world} ranks")
        if K % 2:
            raise ValueError("K must be even (the expert id takes two bf16 columns)")
        self.world, self.rank, self.group = world, rank, group
        self.n_local = n_expert // world
        self.t_loc = n_tok // world
        self.top_k, self.K = top_k, K
        self.cap = self.t_loc * top_k          # rows one source can send one destination
        R = world * self.cap
        # Send/receive rows: K bf16 activations + one int32 expert id.
        self.send = torch.empty(R, K + 2, dtype=torch.bfloat16, device=device)
        self.recv = torch.empty_like(self.send)
        self.y_loc = torch.empty(R, K, dtype=torch.float32, device=device)
        self.y_back = torch.empty_like(self.y_loc)
        self.pos = torch.empty(self.t_loc * top_k, dtype=torch.int32, device=device)
        self.ones = torch.ones(R, 1, dtype=torch.float32, device=device)
        if dispatch is None or combine is None:
            from . import ops
            dispatch = dispatch or ops.ep_dispatch
            combine = combine or ops.ep_combine
        self._dispatch, self._combine = dispatch, combine

    def owner(self, expert):
        return expert // self.n_local

    @staticmethod
    def _ids_view(rows, K):
        """int32 [R, 1] view of the expert-id column of bf16 rows [R, K + 2]."""
        return rows.view(torch.int32)[:, K // 2:K // 2 + 1]

    def send_ids(self):
        return self._ids_view(self.send, self.K)

    def recv_ids(self):
        return self._ids_view(self.recv, self.K)

    def recv_x(self):
        return self.recv[:, :self.K]

    def _exchange(self, out, inp):
        import torch.distributed as dist
        dist.all_to_all_single(out, inp, group=self.group)

    def layer(self, x, ids, w, local_ffn, y):
        """x: [t_loc, K] f32/bf16; ids: int32 [t_loc, top_k] global expert ids;
        w: f32 [t_loc, top_k]; y: f32 [t_loc, K] (written).
        local_ffn(x_rows, local_ids [R, 1], ones [R, 1], out [R, K]) runs this
        rank's experts over the received rows."""
        self._dispatch(ids, x, self.n_local, self.world, self.cap, self.send[:, :self.K],
                       self.send_ids()[:, 0], self.pos)
        self._exchange(self.recv, self.send)
        local_ffn(self.recv_x(), self.recv_ids(), self.ones, self.y_loc)
        self._exchange(self.y_back, self.y_loc)
        self._combine(self.y_back, self.pos, w, y)
        return y
