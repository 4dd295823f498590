"""Sharding a tensor's quantization over GPUs, one process a GPU (torch.distributed).

Expert tensors shard by expert and 2-D tensors by row range; every shard is quantized independently (ggml's blocks
depend on nothing outside their own 256 weights and imatrix row) and owns a contiguous slice of the output bytes,
so the data path needs no collective. The only communication is gathering the byte slices where a caller wants the
whole tensor in one process (all_gather of padded uint8 tensors; over NCCL between GPUs, gloo on the CPU), and the
max-over-ranks of timings.

In-process multi-GPU (one host thread a device, same sharding) is the library's own gpuq_init_devices.
"""


def shard_range(n, rank, world):
    """the contiguous [start, stop) of n units owned by `rank` of `world` (sizes differ by at most one)"""
    base, extra = divmod(int(n), int(world))
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def quantize_sharded(quantize_fn, n_units, unit_bytes, rank, world, group=None, device=None):
    """Quantizes this rank's units with quantize_fn(start, stop) -> uint8 bytes of units [start, stop), then
    gathers every rank's bytes in unit order. Returns the whole tensor's bytes (a torch uint8 tensor on `device`,
    every rank). unit_bytes: output bytes a unit (an expert's or a row's)."""
    import torch
    import torch.distributed as dist
    start, stop = shard_range(n_units, rank, world)
    mine = quantize_fn(start, stop)
    mine = torch.as_tensor(mine, dtype=torch.uint8).reshape(-1).to(device or "cpu")
    if mine.numel() != (stop - start) * unit_bytes:
        raise RuntimeError("rank %d: shard has %d bytes, want %d" % (rank, mine.numel(), (stop - start) * unit_bytes))
    if world == 1:
        return mine
    most = (n_units + world - 1) // world * unit_bytes
    buf = torch.zeros(most, dtype=torch.uint8, device=mine.device)
    buf[:mine.numel()] = mine
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf, group=group)
    out = []
    for r in range(world):
        a, b = shard_range(n_units, r, world)
        out.append(parts[r][:(b - a) * unit_bytes])
    return torch.cat(out)
