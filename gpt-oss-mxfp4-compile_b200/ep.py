"""Expert parallelism: one process per GPU, the experts sharded by contiguous ranges.

The reference runs on one GPU only ("Expert parallelism not implemented",
kernels/cutlass_matmul_investigations.md:231). Here rank r of W owns experts
[r*E/W, (r+1)*E/W); tokens stay data parallel (each rank routes its own tokens). One
forward is

  1. dispatch kernels: stable sort of the T*k assignments by destination rank and FP8
     quantisation of each assignment's hidden row into a packed send row
     [codes H | UE8M0 scales H/32 | pad | local expert i32 | weight f32];
  2. all_to_all_single of the per-rank counts, one device->host read of the splits,
     all_to_all_single of the rows (NCCL over NVLink / NVSwitch);
  3. the local expert forward on the received rows (route sort by local expert, scales
     gathered into the blocked layout, GEMM1 + SwiGLU + requant, GEMM2 + bias x weight),
     one weighted bf16 row back per received row;
  4. all_to_all_single of those rows with the splits reversed;
  5. combine: each token's k rows summed in fp32 in ascending expert order and rounded
     to bf16 once, what the single-device scatter_add_ of bf16 rows gives on the CPU
     (kernels/cutlass_experts.py:445-450).

Quantisation is per row, so the FP8 codes and scales equal the single-GPU ones bit for
bit; rows are independent through both GEMMs.

Two exchange layouts:
  * exact splits (default): rows are compact; the split sizes are read on the host once
    per forward (step 2), so the forward is not CUDA-graph capturable;
  * fixed capacity (`capacity_tokens` set, the same on every rank): every rank sends W
    segments of capacity_tokens*k rows, unused rows marked empty, so both all-to-alls
    have equal splits, nothing is read on the host and the forward can be captured in a
    CUDA graph. It moves W*capacity_tokens*k rows per rank and direction, which pays at
    decode-sized batches where a host round trip costs more than the padding.
The kernels sit behind :class:`CudaKernels`; a different object with the same three
methods can stand in for it (the CPU tests use the oracle's restatement with the gloo
backend).

transport="p2p" (fixed capacity) replaces both all-to-alls with stores into peer-mapped
buffers on the same node: the dispatch kernel quantises each row straight into the
owner's receive buffer and the owner copies each output row straight into the source's
return buffer, each followed by an epoch flag the consumer waits on (csrc/ep_p2p.cuh).
"""
from __future__ import annotations

import types

import torch
import torch.distributed as dist
from torch import nn

from . import ops as _ops
from .cutlass_experts import CutlassGptOssExperts


class CudaKernels:
    """The sm_100a kernels of the three local steps."""

    @staticmethod
    def dispatch(hidden, router_indices, routing_weights, num_experts: int, world_size: int, capacity: int = 0):
        return _ops.ep_dispatch(hidden, router_indices, routing_weights, num_experts, world_size, capacity)

    @staticmethod
    def expert_forward(recv_rows, experts: CutlassGptOssExperts):
        return _ops.ep_expert_forward(recv_rows, experts.gate_up_proj_data, experts.gate_up_proj_scales,
                                      experts.gate_up_proj_bias.data, experts.down_proj_data,
                                      experts.down_proj_scales, experts.down_proj_bias.data, float(experts.alpha),
                                      float(experts.limit), int(experts.gemm_mode))

    @staticmethod
    def combine(back_rows, pos_of, router_indices):
        return _ops.ep_combine(back_rows, pos_of, router_indices)


def shard_experts(experts: CutlassGptOssExperts, rank: int, world_size: int) -> CutlassGptOssExperts:
    """A CutlassGptOssExperts holding experts [rank*E/W, (rank+1)*E/W) of `experts`
    (views of its buffers, no copy)."""
    E = experts.num_experts
    if E % world_size != 0:
        raise ValueError(f"num_experts {E} is not a multiple of world_size {world_size}")
    e_loc = E // world_size
    lo, hi = rank * e_loc, (rank + 1) * e_loc
    cfg = types.SimpleNamespace(num_local_experts=e_loc, intermediate_size=experts.intermediate_size,
                                hidden_size=experts.hidden_size, swiglu_limit=experts.limit)
    loc = CutlassGptOssExperts(cfg).to(experts.gate_up_proj_bias.device)
    loc.alpha, loc.limit, loc.gemm_mode = experts.alpha, experts.limit, experts.gemm_mode
    loc.gate_up_proj_bias.data = experts.gate_up_proj_bias.data[lo:hi]
    loc.down_proj_bias.data = experts.down_proj_bias.data[lo:hi]
    for name in ("gate_up_proj_data", "gate_up_proj_scales", "down_proj_data", "down_proj_scales"):
        setattr(loc, name, getattr(experts, name)[lo:hi])
    return loc


class P2PExchange:
    """The peer-mapped exchange buffers of one expert-parallel group (layout and protocol
    in csrc/ep_p2p.cuh): this rank's buffer is allocated here, every other rank's buffer
    is mapped through its IPC handle (gathered with torch.distributed over the group's
    host-side object collective), and the W base addresses go to the device."""

    def __init__(self, world_size: int, rank: int, capacity: int, hidden_size: int, device, group=None):
        self.world_size, self.rank, self.capacity, self.group = world_size, rank, capacity, group
        nbytes = _ops.ep_p2p_buffer_bytes(world_size, capacity, hidden_size)
        if nbytes <= 0:
            raise ValueError("p2p exchange: bad world_size / capacity / hidden size")
        self.local, handle = _ops.ipc_alloc(nbytes)
        handles = [None] * world_size
        dist.all_gather_object(handles, handle, group=group)
        self.peers = [self.local if r == rank else _ops.ipc_open(handles[r]) for r in range(world_size)]
        self.peer_bases = torch.tensor(self.peers, dtype=torch.int64, device=device)
        self.epoch = 0
        dist.barrier(group=group)               # every rank has mapped every buffer

    def close(self):
        if self.local is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)          # nobody writes into a buffer about to go away
        for r, ptr in enumerate(self.peers):
            if r != self.rank:
                _ops.ipc_close(ptr)
        _ops.ipc_free(self.local)
        self.local = None


class ExpertParallelExperts(nn.Module):
    """Drop-in for CutlassGptOssExperts.forward across a process group: same
    (hidden_states, router_indices, routing_weights) -> out contract, router_indices
    holding GLOBAL expert ids; `local_experts` holds this rank's E/W experts."""

    def __init__(self, local_experts: CutlassGptOssExperts, num_experts: int, group=None, kernels=None,
                 capacity_tokens: int | None = None, transport: str = "nccl", top_k: int = 4):
        super().__init__()
        self.capacity_tokens = capacity_tokens
        if transport not in ("nccl", "p2p"):
            raise ValueError(f"transport must be 'nccl' or 'p2p', got {transport!r}")
        if transport == "p2p" and not capacity_tokens:
            raise ValueError("the p2p transport needs capacity_tokens (fixed-size peer buffers)")
        self.transport = transport
        self.top_k = top_k
        self.group = group
        self.world_size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if local_experts.num_experts * self.world_size != num_experts:
            raise ValueError(f"{local_experts.num_experts} local experts x {self.world_size} ranks != {num_experts}")
        self.experts = local_experts
        self.num_experts = num_experts
        self.hidden_size = local_experts.hidden_size
        self.kernels = kernels if kernels is not None else CudaKernels()
        self.last_splits = None        # exact splits: (send, recv) rows per peer of the last forward
        self.last_send_counts = None   # fixed capacity: device tensor of rows per destination
        self.exchange = None
        if transport == "p2p":
            dev = local_experts.gate_up_proj_bias.device
            cap = capacity_tokens * top_k
            self.exchange = P2PExchange(self.world_size, self.rank, cap, self.hidden_size, dev, group)
            R = self.world_size * cap
            e_loc = local_experts.num_experts
            self._back = torch.empty((R, self.hidden_size), dtype=torch.bfloat16, device=dev)
            nbytes = _ops.workspace_bytes(R, 1, e_loc, self.hidden_size, local_experts.intermediate_size)
            self._ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev)

    def close(self):
        """Release the peer buffers (collective over the group)."""
        if self.exchange is not None:
            self.exchange.close()
            self.exchange = None

    def _p2p_one_launch(self, h, cap: int) -> bool:
        """Decode-sized steps run as one persistent launch (ops.ep_p2p_layer_forward). The
        choice depends only on the group's common sizes (capacity, not this rank's token
        count), so every rank makes the same one."""
        x = self.experts
        return _ops.ep_p2p_layer_fits(self.capacity_tokens, self.top_k, self.num_experts, self.world_size,
                                      self.hidden_size, x.intermediate_size, cap)

    def _p2p_layer(self, h, router_weight, router_bias, idx, w, cap):
        ex, x = self.exchange, self.experts
        out, scores, idx, send_counts, _ = _ops.ep_p2p_layer_forward(
            h, router_weight, router_bias, idx, w, self.top_k, self.num_experts, self.world_size, self.rank,
            x.gate_up_proj_data, x.gate_up_proj_scales, x.gate_up_proj_bias, x.down_proj_data, x.down_proj_scales,
            x.down_proj_bias, cap, ex.local, ex.peer_bases, ex.epoch, self._ws, float(x.alpha), float(x.limit))
        self.last_send_counts = send_counts
        return out, scores, idx

    def _p2p_finish(self, h, idx, send_counts, pos_of, cap):
        """Local experts on the received rows, return rows to their senders, combine."""
        ex, x = self.exchange, self.experts
        _ops.ep_p2p_expert_forward(ex.local, self.world_size, self.rank, cap, ex.epoch, x.gate_up_proj_data,
                                   x.gate_up_proj_scales, x.gate_up_proj_bias, x.down_proj_data,
                                   x.down_proj_scales, x.down_proj_bias, self._back, self._ws,
                                   ex.peer_bases, float(x.alpha), float(x.limit), int(x.gemm_mode))
        self.last_send_counts = send_counts
        return _ops.ep_p2p_combine(ex.local, self.world_size, cap, ex.epoch, pos_of, idx, self.hidden_size, h.device)

    def forward_with_router(self, h: torch.Tensor, router_weight: torch.Tensor, router_bias: torch.Tensor):
        """p2p transport: router + dispatch in one call (one launch at decode sizes), then
        the local experts and the combine. h [T, H] bf16 -> (out [T, H], scores [T, k] bf16,
        router_indices [T, k] int64)."""
        if self.transport != "p2p":
            raise RuntimeError("forward_with_router needs the p2p transport")
        if h.shape[0] > self.capacity_tokens:
            raise RuntimeError(f"p2p exchange sized for {self.capacity_tokens} tokens")
        ex = self.exchange
        ex.epoch += 1
        cap = self.capacity_tokens * self.top_k
        if self._p2p_one_launch(h, cap):
            out, scores, idx = self._p2p_layer(h, router_weight, router_bias, None, None, cap)
            return out, scores, idx
        scores, idx, send_counts, pos_of = _ops.ep_p2p_route_dispatch(
            h, router_weight, router_bias, self.top_k, self.world_size, self.rank, cap, ex.local, ex.peer_bases,
            ex.epoch)
        return self._p2p_finish(h, idx, send_counts, pos_of, cap), scores, idx

    def forward(self, hidden_states: torch.Tensor, router_indices: torch.Tensor,
                routing_weights: torch.Tensor) -> torch.Tensor:
        shape = hidden_states.shape
        H = self.hidden_size
        h = hidden_states.reshape(-1, H).contiguous()
        idx = router_indices.reshape(h.shape[0], router_indices.shape[-1]).contiguous()
        w = routing_weights.reshape(idx.shape).to(torch.float32).contiguous()
        k, g = self.kernels, self.group
        if self.transport == "p2p":
            if h.shape[0] > self.capacity_tokens or idx.shape[1] != self.top_k:
                raise RuntimeError(f"p2p exchange sized for {self.capacity_tokens} tokens x top-{self.top_k}")
            ex = self.exchange
            ex.epoch += 1
            cap = self.capacity_tokens * self.top_k
            if self._p2p_one_launch(h, cap):
                return self._p2p_layer(h, None, None, idx, w, cap)[0].view(shape)
            send_counts, pos_of = _ops.ep_p2p_dispatch(h, idx, w, self.num_experts, self.world_size, self.rank, cap,
                                                       ex.local, ex.peer_bases, ex.epoch)
            return self._p2p_finish(h, idx, send_counts, pos_of, cap).view(shape)
        if self.capacity_tokens:
            if h.shape[0] > self.capacity_tokens:
                raise RuntimeError(f"{h.shape[0]} tokens exceed capacity_tokens={self.capacity_tokens}")
            cap = self.capacity_tokens * idx.shape[1]
            send_rows, send_counts, pos_of = k.dispatch(h, idx, w, self.num_experts, self.world_size, cap)
            recv_rows = torch.empty_like(send_rows)
            dist.all_to_all_single(recv_rows, send_rows, group=g)
            back = k.expert_forward(recv_rows, self.experts)
            ret = torch.empty_like(back)
            dist.all_to_all_single(ret, back, group=g)
            self.last_send_counts = send_counts
            return k.combine(ret, pos_of, idx).view(shape)
        send_rows, send_counts, pos_of = k.dispatch(h, idx, w, self.num_experts, self.world_size)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=g)
        splits = torch.stack([send_counts, recv_counts]).cpu()       # the one device -> host read
        s_send, s_recv = splits[0].tolist(), splits[1].tolist()
        self.last_splits = (s_send, s_recv)
        recv_rows = send_rows.new_empty((sum(s_recv), send_rows.shape[1]))
        dist.all_to_all_single(recv_rows, send_rows, output_split_sizes=s_recv, input_split_sizes=s_send, group=g)
        back = k.expert_forward(recv_rows, self.experts)
        ret = back.new_empty((send_rows.shape[0], H))
        dist.all_to_all_single(ret, back, output_split_sizes=s_send, input_split_sizes=s_recv, group=g)
        out = k.combine(ret, pos_of, idx)
        return out.view(shape)


class ExpertParallelMoELayer(nn.Module):
    """Router (local tokens) + expert-parallel experts: the GptOssMLP shape of the block
    with the experts sharded. `router_weight` [E, H] / `router_bias` [E] bf16 are
    replicated on every rank."""

    def __init__(self, router_weight: torch.Tensor, router_bias: torch.Tensor, top_k: int,
                 experts: ExpertParallelExperts, router=None):
        """`router(hidden, weight, bias, top_k) -> (logits, scores, indices)` replaces the
        fused router op when given (the host-side tests pass the CPU router)."""
        super().__init__()
        self.router_weight = nn.Parameter(router_weight, requires_grad=False)
        self.router_bias = nn.Parameter(router_bias, requires_grad=False)
        self.top_k = top_k
        self.experts = experts
        self._router = router

    def forward(self, hidden_states: torch.Tensor):
        h = hidden_states.reshape(-1, self.experts.hidden_size).contiguous()
        if self._router is not None:
            _, scores, idx = self._router(h, self.router_weight.data, self.router_bias.data, int(self.top_k))
            out = self.experts(h, idx, scores.float())
            return out.view(hidden_states.shape), scores, idx
        _ops.register_ops()
        if self.experts.transport == "p2p" and self.top_k == self.experts.top_k:
            out, scores, idx = self.experts.forward_with_router(h, self.router_weight, self.router_bias)
            return out.view(hidden_states.shape), scores, idx
        _, scores, idx = torch.ops.gptoss.router_topk(h, self.router_weight.data, self.router_bias.data,
                                                      int(self.top_k))
        out = self.experts(h, idx, scores.float())
        return out.view(hidden_states.shape), scores, idx


__all__ = ["CudaKernels", "ExpertParallelExperts", "ExpertParallelMoELayer", "shard_experts"]
