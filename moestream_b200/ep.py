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
  3. the local FFN over the received rows with top_k = 1 and no weighting
     (unused rows land in the zero slot and give exact zeros);
  4. one equal-split all-to-all of the f32 results back to the source ranks;
  5. combine: y[t] = sum_k w[t, k] * (row of pair (t, k)), k ascending.

Two transports carry steps 1-2 and 4:
  - "collective": the library's packing kernels around
    torch.distributed.all_to_all_single (NCCL on GPUs, gloo on CPU);
    dispatch and combine may be replaced by any functions with the same
    meaning (the CPU tests pass the oracle's);
  - "peers": kernels that store the rows straight into the other GPUs'
    exchange buffers over NVLink and raise a flag there; the receiving rank
    waits on its flags (bounded) before reading. No collective runs in the
    layer, and every launch can be captured in a CUDA graph.
"""
import ctypes

import torch


class _DeviceBytes:
    """Device memory owned elsewhere, seen by torch through the CUDA array
    interface."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3,
                                         "strides": None}


class ExpertParallel:
    """Buffers and steps of one rank's expert-parallel MoE layer."""

    def __init__(self, world, rank, n_expert, n_tok, top_k, K, device, group=None,
                 dispatch=None, combine=None, transport="collective"):
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
        self.transport = transport
        self.y_loc = torch.empty(R, K, dtype=torch.float32, device=device)
        self.pos = torch.empty(self.t_loc * top_k, dtype=torch.int32, device=device)
        self._buf, self._opened = None, []
        if transport == "peers":
            self._open_peers(device)
        elif transport == "collective":
            # Send/receive rows: K bf16 activations + one int32 expert id.
            self.row_elems = K + 2
            self.send = torch.empty(R, K + 2, dtype=torch.bfloat16, device=device)
            self.recv = torch.empty_like(self.send)
            self.y_back = torch.empty_like(self.y_loc)
        else:
            raise ValueError(f"unknown transport {transport!r}")
        self.route = None
        if dispatch is None or combine is None:
            from . import ops
            dispatch = dispatch or ops.ep_dispatch
            combine = combine or ops.ep_combine
            self.route = ops.RouteBuffers(R, self.n_local, device)
        self._dispatch, self._combine = dispatch, combine

    def _open_peers(self, device):
        """Creates this rank's exchange buffer, shares its IPC handle with the
        other ranks (an all-gather on the process group) and maps theirs."""
        import torch.distributed as dist

        from ._lib import EP_HANDLE_BYTES, EpPeers, check, lib
        L = lib()
        R = self.world * self.cap
        nbytes = int(L.msb_ep_buffer_bytes(self.world, self.cap, self.K))
        if nbytes <= 0:
            raise ValueError("expert-parallel peer buffer: unsupported shape")
        buf = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * EP_HANDLE_BYTES)()
        check(L.msb_ep_buffer_create(nbytes, ctypes.byref(buf), handle))
        self._buf = buf.value
        mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=device)
        every = torch.empty(self.world * EP_HANDLE_BYTES, dtype=torch.uint8, device=device)
        dist.all_gather_into_tensor(every, mine, group=self.group)
        every = every.cpu().tolist()
        peers = EpPeers()
        peers.n_rank, peers.rank, peers.cap, peers.K = self.world, self.rank, self.cap, self.K
        for r in range(self.world):
            if r == self.rank:
                peers.peer[r] = self._buf
                continue
            h = (ctypes.c_uint8 * EP_HANDLE_BYTES)(*every[r * EP_HANDLE_BYTES:
                                                         (r + 1) * EP_HANDLE_BYTES])
            p = ctypes.c_void_p()
            check(L.msb_ep_buffer_open(h, ctypes.byref(p)))
            self._opened.append(p.value)
            peers.peer[r] = p.value
        self.peers = peers
        row_bytes = int(L.msb_ep_row_bytes(self.K))
        self.row_elems = row_bytes // 2
        self.recv = torch.as_tensor(_DeviceBytes(self._buf, (R, self.row_elems), "<i2"),
                                    device=device).view(torch.bfloat16)
        off = int(L.msb_ep_yback_offset(self.world, self.cap, self.K))
        self.y_back = torch.as_tensor(_DeviceBytes(self._buf + off, (R, self.K), "<f4"),
                                      device=device)

    def close(self):
        """Unmaps the peers' buffers and frees this rank's (peers transport);
        every rank must call it, after its last layer."""
        if self._buf is None:
            return
        import torch.distributed as dist

        from ._lib import check, lib
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for p in self._opened:
            check(lib().msb_ep_buffer_close(ctypes.c_void_p(p)))
        self._opened = []
        dist.barrier(group=self.group)
        self.recv = self.y_back = None
        check(lib().msb_ep_buffer_destroy(ctypes.c_void_p(self._buf)))
        self._buf = None

    def owner(self, expert):
        return expert // self.n_local

    @staticmethod
    def _ids_view(rows, K):
        """int32 [R, 1] view of the expert-id column (after K bf16 values)."""
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

    def layer(self, x, ids, w, local_ffn, y, pools=None):
        """x: [t_loc, K] f32/bf16; ids: int32 [t_loc, top_k] global expert ids;
        w: f32 [t_loc, top_k]; y: f32 [t_loc, K] (written).
        local_ffn(x_rows [R, K], local_ids [R, 1], route, out [R, K]) runs this
        rank's experts over the received rows with top_k 1 and no weighting;
        `route` is those rows grouped by local slot (RouteBuffers) on GPUs,
        None when dispatch and combine were passed in.
        pools (peers transport): (gate, up, down, up_row0, workspace) of this
        rank's experts; where the tensor cores take them, the down projection
        returns its rows to their source ranks itself and local_ffn is not
        called."""
        if self.transport == "peers":
            from . import ops
            ops.ep_dispatch_peers(self.peers, ids, x, self.n_local, self.pos)
            route = ops.ep_remap_group(self.peers, self.n_local, self.route)
            fused = False
            if pools is not None:
                gate, up, down, up_row0, ws = pools
                fused = ops.ep_moe_ffn_peers(self.peers, gate, up, down, route, ws, up_row0)
            if not fused:
                local_ffn(self.recv_x(), self.recv_ids(), route, self.y_loc)
                ops.ep_return_peers(self.peers, self.y_loc)
            ops.ep_combine_peers(self.peers, self.pos, w, y)
            return y
        self._dispatch(ids, x, self.n_local, self.world, self.cap, self.send[:, :self.K],
                       self.send_ids()[:, 0], self.pos)
        self._exchange(self.recv, self.send)
        route = None
        if self.route is not None:
            from . import ops
            route = ops.remap_group(self.recv_ids(), self.n_local, route=self.route)
        local_ffn(self.recv_x(), self.recv_ids(), route, self.y_loc)
        self._exchange(self.y_back, self.y_loc)
        self._combine(self.y_back, self.pos, w, y)
        return y
