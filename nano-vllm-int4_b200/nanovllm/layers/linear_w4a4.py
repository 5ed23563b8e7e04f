"""W4A4 linear layers: activation prep (RHT + INT4 quantisation) + grouped INT4 GEMM.

``W4A4Linear`` is the drop-in for ``nanovllm/layers/linear_w4a4.py:15-36`` of
the reference: same constructor, buffer names, dtypes and shapes
(``packed_weight`` int8 [N, K/2], ``weight_scale`` bf16 [N, K/128], ``signs``
int8 [K]), same forward (two launches, two small allocations that come from
the CUDA-graph pool when captured).  Its defaults reproduce the reference
checkpoint contract (layout ``row_DH_paley12_kron_sylvester_v1``, codes in
[-7, 7]); ``layout="block128", clamp_lo=-8`` selects the block-diagonal layout
and full INT4 range of the benchmark configurations.

Tensor parallelism is new relative to the reference (which refuses it for
W4A4, ``linear_w4a4.py:18-19``).  The classes below follow the BF16 pattern of
``nanovllm/layers/linear.py:54-155``:

* ``W4A4ColumnParallelLinear`` / ``W4A4MergedColumnParallelLinear`` /
  ``W4A4QKVParallelLinear`` shard the output dimension N.  Every rank holds the
  full sign vector and quantises the (replicated) input itself; no
  communication.
* ``W4A4RowParallelLinear`` shards K on 128-group boundaries.  With the
  ``block128`` layout the transform and quantisation of a K shard need only
  that shard, so each rank runs the GEMM on its groups into FP32 and the
  partial outputs are summed with one all-reduce over NVLink (NCCL).  The
  full-width checkpoint layout mixes all of K, so row-parallel ranks first
  all-gather the BF16 input, quantise the whole row and keep their groups.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
from torch import nn

from nanovllm.kernels.rht_a4_tilelang import (LAYOUT_VERSION, add_rmsnorm_rht_quant_i8, rht_quant_i8,
                                               silu_mul_rht_quant_i8)
from nanovllm.kernels.w4a4_grouped_kernel import w4a4_grouped_gemm_i8
from nanovllm import _native

BLOCK128 = "block128"


def _tp(tp_rank, tp_size):
    if tp_size is None:
        tp_size = dist.get_world_size() if dist.is_initialized() else 1
    if tp_rank is None:
        tp_rank = dist.get_rank() if dist.is_initialized() else 0
    return tp_rank, tp_size


def _divide(numerator, denominator):
    if numerator % denominator:
        raise ValueError(f"{numerator} is not divisible by {denominator}")
    return numerator // denominator


class W4A4Linear(nn.Module):
    def __init__(self, input_size: int, output_size: int, bias: bool = False, *, layout=LAYOUT_VERSION,
                 clamp_lo: int = -7):
        super().__init__()
        if type(self) is W4A4Linear and dist.is_initialized() and dist.get_world_size() != 1:
            raise ValueError("W4A4Linear supports one GPU only; use the W4A4*ParallelLinear classes")
        self.layout_id = _native.LAYOUTS[layout] if isinstance(layout, str) else int(layout)
        if bias or output_size % 8:
            raise ValueError("W4A4 requires bias-free Qwen3-8B projection shapes")
        if self.layout_id == _native.LAYOUT_ROW_DH and input_size not in (4096, 12288):
            raise ValueError("W4A4 requires bias-free Qwen3-8B projection shapes")
        if input_size % 128:
            raise ValueError("W4A4 requires K divisible by 128")
        if clamp_lo not in (-7, -8):
            raise ValueError("clamp_lo must be -7 or -8")
        self.layout = layout
        self.clamp_lo = clamp_lo
        self.in_features, self.out_features = input_size, output_size
        self.register_buffer("packed_weight", torch.empty(output_size, input_size // 2, dtype=torch.int8))
        self.register_buffer("weight_scale", torch.empty(output_size, input_size // 128, dtype=torch.bfloat16))
        self.register_buffer("signs", torch.empty(input_size, dtype=torch.int8))

    def quantize_input(self, flat: torch.Tensor):
        """Activation prep into the GEMM-ready INT8 layout: (codes [M,K], scales [M,K/128])."""
        m, k = flat.shape
        codes = torch.empty((m, k), dtype=torch.int8, device=flat.device)
        scale = torch.empty((m, k // 128), dtype=torch.bfloat16, device=flat.device)
        rht_quant_i8(flat, self.signs, out_codes=codes, out_scale=scale, layout=self.layout_id,
                     clamp_lo=self.clamp_lo)
        return codes, scale

    def quantize_silu_mul_input(self, gate_up: torch.Tensor):
        """The activation prep of SiluAndMul(gate_up) fused with it (the MLP's
        down projection): gate_up [M, 2K] -> (codes [M,K], scales [M,K/128])."""
        m = gate_up.shape[0]
        codes = torch.empty((m, self.in_features), dtype=torch.int8, device=gate_up.device)
        scale = torch.empty((m, self.in_features // 128), dtype=torch.bfloat16, device=gate_up.device)
        silu_mul_rht_quant_i8(gate_up, self.signs, out_codes=codes, out_scale=scale, layout=self.layout_id,
                              clamp_lo=self.clamp_lo)
        return codes, scale

    def _gemm(self, codes, scale):
        return w4a4_grouped_gemm_i8(codes, self.packed_weight, scale, self.weight_scale)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape[-1] != self.in_features or x.dtype != torch.bfloat16:
            raise ValueError("W4A4Linear requires BF16 activations with the configured input width")
        flat = x.reshape(-1, self.in_features).contiguous()
        codes, scale = self.quantize_input(flat)
        return self._gemm(codes, scale).reshape(*x.shape[:-1], self.out_features)

    def forward_add_rmsnorm(self, x: torch.Tensor, residual, norm_weight: torch.Tensor, eps: float = 1e-6):
        """``self(RMSNorm(x + residual))`` with the decoder layer's add + RMSNorm
        fused into the prep (layernorm.py:33-45, then this projection): returns
        ``(output, new_residual)`` with new_residual = bf16(x + residual), or
        ``(output, x)`` when ``residual`` is None (rms_forward on x)."""
        if x.shape[-1] != self.in_features or x.dtype != torch.bfloat16:
            raise ValueError("forward_add_rmsnorm requires BF16 activations with the configured input width")
        flat = x.reshape(-1, self.in_features).contiguous()
        m = flat.shape[0]
        codes = torch.empty((m, self.in_features), dtype=torch.int8, device=flat.device)
        scale = torch.empty((m, self.in_features // 128), dtype=torch.bfloat16, device=flat.device)
        res = None if residual is None else residual.reshape(-1, self.in_features).contiguous()
        new_res = torch.empty_like(flat) if res is not None else None
        add_rmsnorm_rht_quant_i8(flat, res, norm_weight, eps, self.signs, out_codes=codes, out_scale=scale,
                                 out_residual=new_res, layout=self.layout_id, clamp_lo=self.clamp_lo)
        out = self._gemm(codes, scale).reshape(*x.shape[:-1], self.out_features)
        return out, (x if new_res is None else new_res.reshape(x.shape))

    def forward_silu_mul(self, gate_up: torch.Tensor) -> torch.Tensor:
        """``self(SiluAndMul()(gate_up))`` with the activation fused into the
        prep (Qwen3MLP.forward's act_fn + down_proj): gate_up BF16 [..., 2K]."""
        if gate_up.shape[-1] != 2 * self.in_features or gate_up.dtype != torch.bfloat16:
            raise ValueError("forward_silu_mul requires BF16 gate/up activations of width 2K")
        flat = gate_up.reshape(-1, 2 * self.in_features).contiguous()
        codes, scale = self.quantize_silu_mul_input(flat)
        return self._gemm(codes, scale).reshape(*gate_up.shape[:-1], self.out_features)

    @torch.no_grad()
    def load_full(self, packed: torch.Tensor, scale: torch.Tensor, signs: torch.Tensor) -> None:
        """Copy unsharded checkpoint tensors (packed [N,K/2], scale [N,K/128], signs [K])."""
        self.packed_weight.copy_(packed)
        self.weight_scale.copy_(scale)
        self.signs.copy_(signs)


class W4A4ColumnParallelLinear(W4A4Linear):
    """Output dimension sharded over the TP group (linear.py:54-73 pattern)."""

    def __init__(self, input_size: int, output_size: int, bias: bool = False, *, layout=BLOCK128,
                 clamp_lo: int = -8, tp_rank=None, tp_size=None):
        self.tp_rank, self.tp_size = _tp(tp_rank, tp_size)
        self.full_output_size = output_size
        super().__init__(input_size, _divide(output_size, self.tp_size), bias, layout=layout, clamp_lo=clamp_lo)

    def _rows(self, full_rows: int):
        size = _divide(full_rows, self.tp_size)
        return self.tp_rank * size, size

    @torch.no_grad()
    def load_full(self, packed, scale, signs):
        start, size = self._rows(packed.shape[0])
        self.packed_weight.copy_(packed.narrow(0, start, size))
        self.weight_scale.copy_(scale.narrow(0, start, size))
        self.signs.copy_(signs)


class W4A4MergedColumnParallelLinear(W4A4ColumnParallelLinear):
    """Several column blocks (e.g. gate and up) concatenated along N, each sharded
    separately so that every rank holds matching slices (linear.py:76-93)."""

    def __init__(self, input_size: int, output_sizes: list[int], bias: bool = False, **kw):
        self.output_sizes = list(output_sizes)
        super().__init__(input_size, sum(output_sizes), bias, **kw)

    @torch.no_grad()
    def load_shard(self, shard_id: int, packed, scale):
        offset = sum(self.output_sizes[:shard_id]) // self.tp_size
        size = self.output_sizes[shard_id] // self.tp_size
        self.packed_weight.narrow(0, offset, size).copy_(packed.chunk(self.tp_size, 0)[self.tp_rank])
        self.weight_scale.narrow(0, offset, size).copy_(scale.chunk(self.tp_size, 0)[self.tp_rank])

    @torch.no_grad()
    def load_full(self, packed, scale, signs):
        start = 0
        for i, n in enumerate(self.output_sizes):
            self.load_shard(i, packed.narrow(0, start, n), scale.narrow(0, start, n))
            start += n
        self.signs.copy_(signs)


class W4A4QKVParallelLinear(W4A4ColumnParallelLinear):
    """Fused q/k/v projection sharded by heads (linear.py:96-128)."""

    def __init__(self, hidden_size: int, head_size: int, total_num_heads: int, total_num_kv_heads=None,
                 bias: bool = False, **kw):
        tp_rank, tp_size = _tp(kw.get("tp_rank"), kw.get("tp_size"))
        total_num_kv_heads = total_num_kv_heads or total_num_heads
        self.head_size = head_size
        self.total_num_heads, self.total_num_kv_heads = total_num_heads, total_num_kv_heads
        self.num_heads = _divide(total_num_heads, tp_size)
        self.num_kv_heads = _divide(total_num_kv_heads, tp_size)
        super().__init__(hidden_size, (total_num_heads + 2 * total_num_kv_heads) * head_size, bias, **kw)

    @torch.no_grad()
    def load_shard(self, shard_id: str, packed, scale):
        if shard_id not in ("q", "k", "v"):
            raise ValueError(shard_id)
        q = self.num_heads * self.head_size
        kv = self.num_kv_heads * self.head_size
        offset, size = {"q": (0, q), "k": (q, kv), "v": (q + kv, kv)}[shard_id]
        self.packed_weight.narrow(0, offset, size).copy_(packed.chunk(self.tp_size, 0)[self.tp_rank])
        self.weight_scale.narrow(0, offset, size).copy_(scale.chunk(self.tp_size, 0)[self.tp_rank])

    @torch.no_grad()
    def load_full(self, packed, scale, signs):
        q = self.total_num_heads * self.head_size
        kv = self.total_num_kv_heads * self.head_size
        for sid, (start, n) in zip("qkv", ((0, q), (q, kv), (q + kv, kv))):
            self.load_shard(sid, packed.narrow(0, start, n), scale.narrow(0, start, n))
        self.signs.copy_(signs)


# One peer buffer per (process group, device), shared by every row-parallel
# layer of the group: outputs of up to PEER_CAPACITY elements (32 tokens x 8192).
PEER_CAPACITY = 32 * 8192
_PEER_STATE = {}  # (id(group), device index) -> (group, rank, every rank's buffer address), or False (NCCL only)


def _setup_peer(group, rank, world, device):
    """Allocate this rank's peer buffer, exchange IPC handles over the group and
    open the others'.  Returns every rank's buffer address, or False when any
    rank could not (then every rank keeps the NCCL all-reduce)."""
    own, handle = None, bytes(_native.IPC_HANDLE_BYTES)
    try:
        own, handle = _native.peer_buffer_alloc(PEER_CAPACITY, device)
    except (RuntimeError, ValueError):
        pass
    mine = torch.tensor(list(handle) + [0 if own is None else 1], dtype=torch.uint8, device=device)
    every = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(every, mine, group=group)
    rows = [bytes(t.cpu().tolist()) for t in every]
    opened, ok = {}, all(r[-1] == 1 for r in rows)
    if ok:
        try:
            for r, row in enumerate(rows):
                if r != rank:
                    opened[r] = _native.peer_buffer_open(row[:-1], device)
        except (RuntimeError, ValueError):
            ok = False
    flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=device)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
    if int(flag.item()) == 1:
        return group, rank, [own if r == rank else opened[r] for r in range(world)]
    for addr in opened.values():
        _native.peer_buffer_close(addr, device)
    if own is not None:
        _native.peer_buffer_free(own, device)
    return False


def release_peer_buffers():
    """Close the peers' buffers and free this rank's (collective: every rank
    calls it after its last forward, once no CUDA graph that uses the buffers
    will be replayed).  Barriers keep a rank from freeing its buffer while a
    peer's last all-reduce may still be writing into it."""
    for (_, index), state in list(_PEER_STATE.items()):
        if state:
            group, rank, addrs = state
            device = torch.device("cuda", index)
            torch.cuda.synchronize(device)
            dist.barrier(group=group)
            for r, addr in enumerate(addrs):
                if r != rank:
                    _native.peer_buffer_close(addr, device)
            dist.barrier(group=group)
            _native.peer_buffer_free(addrs[rank], device)
    _PEER_STATE.clear()


class W4A4RowParallelLinear(W4A4Linear):
    """Input dimension K sharded on 128-group boundaries; partial outputs summed
    in FP32 with one all-reduce (linear.py:131-155 pattern).

    Up to PEER_MAX_TOKENS rows the sum runs over NVLink peer memory: by
    default (``fuse_peer_gemm``) the GEMM's CTAs store their FP32 output tiles
    straight into every rank's inbox and a small kernel adds the ranks' tiles
    in rank order to BF16; with ``fuse_peer_gemm = False`` the GEMM writes its
    partial into this rank's peer buffer and the one-shot all-reduce kernel
    exchanges and sums it.  Both give the same BF16 on every rank and save the
    NCCL launch and latency (about 14 us per call at decode sizes).  The peer
    buffers are set up on the first forward outside a
    CUDA-graph capture (one all-gather of IPC handles over the group); if any
    rank cannot set them up, every rank keeps the NCCL all-reduce.  Larger
    batches use NCCL."""

    PEER_MAX_TOKENS = 32

    def __init__(self, input_size: int, output_size: int, bias: bool = False, *, layout=BLOCK128,
                 clamp_lo: int = -8, tp_rank=None, tp_size=None, group=None):
        self.tp_rank, self.tp_size = _tp(tp_rank, tp_size)
        self.group = group
        self.full_input_size = input_size
        k_local = _divide(input_size, self.tp_size)
        if k_local % 128:
            raise ValueError("row-parallel K shards must be whole 128-groups")
        lid = _native.LAYOUTS[layout] if isinstance(layout, str) else int(layout)
        self.gather_input = lid == _native.LAYOUT_ROW_DH and self.tp_size > 1
        # With the full-width layout the module quantises the gathered row, so its
        # signs buffer covers all of K; the weights cover this rank's K shard.
        nn.Module.__init__(self)
        self.layout, self.layout_id, self.clamp_lo = layout, lid, clamp_lo
        if bias or output_size % 8 or clamp_lo not in (-7, -8):
            raise ValueError("W4A4 requires bias-free projection shapes")
        if lid == _native.LAYOUT_ROW_DH and input_size not in (4096, 12288):
            raise ValueError("W4A4 requires bias-free Qwen3-8B projection shapes")
        self.in_features, self.out_features = k_local, output_size
        self.register_buffer("packed_weight", torch.empty(output_size, k_local // 2, dtype=torch.int8))
        self.register_buffer("weight_scale", torch.empty(output_size, k_local // 128, dtype=torch.bfloat16))
        self.register_buffer("signs", torch.empty(input_size if self.gather_input else k_local, dtype=torch.int8))
        self.use_peer_allreduce = True
        self.fuse_peer_gemm = True
        self._fused_peer_ok = {}  # tokens -> whether the fused peer GEMM can plan this shape

    def _fused_peer_plannable(self, m: int, device) -> bool:
        """Whether the fused peer-memory GEMM has a launch plan for m tokens (its
        grid must fit the per-CTA flag slots).  The plan depends only on the
        shape and the SM count, so every rank of the group decides alike and
        falls back to the same path."""
        ok = self._fused_peer_ok.get(m)
        if ok is None:
            sms = torch.cuda.get_device_properties(device).multi_processor_count
            ok = _native.w4a4_stream_plan(m, self.out_features, self.in_features, _native.GEMM_W_SCALE_GROUPED,
                                          sm_count=sms, peer=True) is not None
            self._fused_peer_ok[m] = ok
        return ok

    def _peer_buffers(self, device):
        """The group's peer buffers, setting them up on first use (collective)."""
        if not self.use_peer_allreduce or device.type != "cuda" or self.tp_size > 8:
            return None
        key = (id(self.group), device.index)
        state = _PEER_STATE.get(key)
        if state is None:
            if torch.cuda.is_current_stream_capturing():
                return None
            state = _setup_peer(self.group, self.tp_rank, self.tp_size, device)
            _PEER_STATE[key] = state
        return state[2] if state else None

    @torch.no_grad()
    def load_full(self, packed, scale, signs):
        k_local = self.in_features
        self.packed_weight.copy_(packed.narrow(1, self.tp_rank * k_local // 2, k_local // 2))
        self.weight_scale.copy_(scale.narrow(1, self.tp_rank * k_local // 128, k_local // 128))
        self.signs.copy_(signs if self.gather_input else signs.narrow(0, self.tp_rank * k_local, k_local))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape[-1] != self.in_features or x.dtype != torch.bfloat16:
            raise ValueError("W4A4RowParallelLinear requires BF16 activations of the local K shard")
        flat = x.reshape(-1, self.in_features).contiguous()
        if self.gather_input:
            parts = [torch.empty_like(flat) for _ in range(self.tp_size)]
            dist.all_gather(parts, flat, group=self.group)
            full = torch.cat(parts, dim=1)
            codes_full, scale_full = W4A4Linear.quantize_input(self, full)
            k_local = self.in_features
            codes = codes_full[:, self.tp_rank * k_local:(self.tp_rank + 1) * k_local].contiguous()
            scale = scale_full[:, self.tp_rank * k_local // 128:(self.tp_rank + 1) * k_local // 128].contiguous()
        else:
            codes, scale = self.quantize_input(flat)
        return self._gemm(codes, scale).reshape(*x.shape[:-1], self.out_features)

    def forward_silu_mul(self, gate_up: torch.Tensor) -> torch.Tensor:
        if self.gather_input:
            raise ValueError("forward_silu_mul needs a shard-local layout (block128) or tp_size 1")
        return W4A4Linear.forward_silu_mul(self, gate_up)

    def _gemm(self, codes, scale):
        """GEMM of this rank's K shard and the sum over the group (BF16 [M, N])."""
        if self.tp_size == 1:
            out = w4a4_grouped_gemm_i8(codes, self.packed_weight, scale, self.weight_scale)
        else:
            m = codes.shape[0]
            count = m * self.out_features
            peers = self._peer_buffers(codes.device) if m <= self.PEER_MAX_TOKENS else None
            if peers and count <= PEER_CAPACITY and self.fuse_peer_gemm and self._fused_peer_plannable(m, codes.device):
                out = torch.empty((m, self.out_features), dtype=torch.bfloat16, device=codes.device)
                _native.w4a4_gemm_peer_allreduce_bf16(codes, self.packed_weight, scale, self.weight_scale, out, peers,
                                                      self.tp_rank, PEER_CAPACITY, _native.GEMM_W_SCALE_GROUPED)
            elif peers and count <= PEER_CAPACITY:
                _native.w4a4_gemm_i8_to(codes, self.packed_weight, scale, self.weight_scale,
                                        peers[self.tp_rank] + _native.peer_header_bytes(),
                                        _native.GEMM_W_SCALE_GROUPED | _native.GEMM_OUT_FP32)
                out = torch.empty((m, self.out_features), dtype=torch.bfloat16, device=codes.device)
                _native.peer_allreduce_bf16(peers, self.tp_rank, out, count, PEER_CAPACITY)
            else:
                partial = w4a4_grouped_gemm_i8(codes, self.packed_weight, scale, self.weight_scale, out_fp32=True)
                dist.all_reduce(partial, group=self.group)
                out = partial.to(torch.bfloat16)
        return out
