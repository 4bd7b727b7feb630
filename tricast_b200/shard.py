"""One emulated GEMM split across the GPUs of a box by N-column slabs (strong scaling).

Every output ``(m, n)`` of TriCast's emulated GEMM is computed independently
(``src/tricast/reference/mma.py:340``), so rank ``r`` of ``g`` takes the weight rows
``[r*N/g, (r+1)*N/g)`` with the whole K (the accumulation order is untouched) and all of the
activations, and produces the output columns of its slab. The slab result is bit-identical to the
same columns of the single-GPU GEMM.

The one exchange the split needs is in the weight quantization: schemes whose scale depends on the
whole weight tensor (NVFP4's global decode scale ``d2``, a per-tensor FP8 scale) need the tensor amax.
Each rank reduces its slab's amax to fp32 bits on the device (``tc_tensor_amax_bits``), one NCCL
all-reduce MAX of that 4-byte word makes it global, and the slab is quantized against it, which gives
exactly the rows of the whole tensor's QTensor. Schemes with only local scales (per group, per row)
need no exchange. The outputs stay sharded; :func:`gather_columns` assembles the full ``[M, N]``
output with one all-gather when a caller wants it.
"""

from __future__ import annotations

import torch

from . import _native as N
from .quantize import quantize_into


def column_slab(n: int, world: int, rank: int) -> tuple[int, int]:
    """Weight rows (output columns) ``[start, end)`` of ``rank``: ``n`` split as evenly as possible,
    the first ``n % world`` ranks taking one extra."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def needs_tensor_amax(spec) -> bool:
    """Whether the scheme's scales depend on the amax of the whole tensor (and on nothing else of it).
    Raises for tensor-granularity schemes whose scale needs more of the whole tensor than its amax
    (zero points, MSE or percentile searches): those do not shard by rows."""
    sf = spec.scale
    if sf is None:
        return False
    if spec.granularity == "tensor":
        if spec.zero_point != "none" or sf.method in ("mse", "percentile"):
            raise ValueError(f"a {sf.method} tensor scale with zero point {spec.zero_point!r} does not shard by rows")
        return True
    return bool(sf.two_level)


def shard_amax(x: torch.Tensor, group=None) -> torch.Tensor:
    """The amax of the whole tensor of which ``x`` is this rank's shard (fp32 scalar on ``x``'s device,
    NaN-propagating). With a process group of more than one rank this is one all-reduce MAX of a
    32-bit word; the bits are those of non-negative floats (NaN above Inf), so the integer max is the
    float max."""
    import torch.distributed as dist

    x2d = x.reshape(-1, x.shape[-1]).contiguous()
    bits = torch.zeros((), dtype=torch.int32, device=x.device)
    with torch.cuda.device(x.device):
        N.check(N.lib().tc_tensor_amax_bits(N.ptr(x2d), N.dtype_code(x2d.dtype), x2d.numel(), N.ptr(bits),
                                            N.stream_of(x.device)), "tc_tensor_amax_bits")
    return reduce_amax_bits(bits, group).view(torch.float32)


def reduce_amax_bits(bits: torch.Tensor, group=None) -> torch.Tensor:
    """Max of every rank's int32 amax bits (in place; one all-reduce when the group has several ranks)."""
    import torch.distributed as dist

    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(bits, op=dist.ReduceOp.MAX, group=group)
    return bits


def quantize_shard(x: torch.Tensor, spec, group=None):
    """Quantize this rank's row shard of a tensor so that it equals those rows of the whole tensor's
    QTensor (deterministic roundings)."""
    if not needs_tensor_amax(spec):
        return quantize_into(x, spec)[0]
    amax = shard_amax(x, group)
    if spec.granularity == "tensor":
        return quantize_into(x, spec, amax=amax)[0]
    return quantize_into(x, spec, tensor_amax=amax)[0]


def quantize_operands(a: torch.Tensor, spec_a, b_shard: torch.Tensor, spec_b, group=None):
    """(QTensor of all of ``a``, QTensor of this rank's shard of ``b``) for one N-column slab of a GEMM.
    When ``b``'s scheme needs the whole tensor's amax, the all-reduce of the shards' amax bits is
    issued asynchronously and ``a`` is quantized while it is in flight."""
    import torch.distributed as dist

    if not needs_tensor_amax(spec_b) or not (dist.is_initialized() and dist.get_world_size(group) > 1):
        return quantize_into(a, spec_a)[0], quantize_shard(b_shard, spec_b, group)
    x2d = b_shard.reshape(-1, b_shard.shape[-1]).contiguous()
    bits = torch.zeros((), dtype=torch.int32, device=b_shard.device)
    with torch.cuda.device(b_shard.device):
        N.check(N.lib().tc_tensor_amax_bits(N.ptr(x2d), N.dtype_code(x2d.dtype), x2d.numel(), N.ptr(bits),
                                            N.stream_of(b_shard.device)), "tc_tensor_amax_bits")
    work = dist.all_reduce(bits, op=dist.ReduceOp.MAX, group=group, async_op=True)
    qa = quantize_into(a, spec_a)[0]
    work.wait()  # the current stream waits for the reduction; the host does not
    amax = bits.view(torch.float32)
    if spec_b.granularity == "tensor":
        return qa, quantize_into(b_shard, spec_b, amax=amax)[0]
    return qa, quantize_into(b_shard, spec_b, tensor_amax=amax)[0]


def gather_columns(slab: torch.Tensor, n: int, group=None) -> torch.Tensor:
    """The full ``[M, n]`` output from every rank's ``[M, slab]`` column slab (one all-gather)."""
    import torch.distributed as dist

    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1:
        return slab
    widths = [column_slab(n, world, r) for r in range(world)]
    most = max(e - s for s, e in widths)
    padded = slab.new_zeros((most, slab.shape[0]))
    padded[: slab.shape[1]] = slab.T
    parts = slab.new_empty((world * most, slab.shape[0]))
    dist.all_gather_into_tensor(parts, padded, group=group)
    parts = parts.view(world, most, slab.shape[0])
    return torch.cat([parts[r, : e - s] for r, (s, e) in enumerate(widths)]).T.contiguous()


__all__ = ["column_slab", "needs_tensor_amax", "shard_amax", "reduce_amax_bits", "quantize_shard", "quantize_operands", "gather_columns"]
