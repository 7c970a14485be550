"""Tensor-parallel model setup over torch.distributed (one process per GPU).

The library does the collectives itself (an in-graph NVLink peer-memory allreduce
after the row-parallel O and down projections, and a cross-rank argmax);
torch.distributed only carries the one-time exchange of the 64-byte CUDA IPC
handles (any backend: gloo on the host is enough)."""
from __future__ import annotations


def shard_ranges(cfg: dict, rank: int, world: int) -> dict:
    """The slices of the global model that `rank` holds (mirrors llama_model_create):
    q heads, KV heads, FFN indices and lm_head rows (vocab split in multiples of 16)."""
    if world <= 1:
        return {"heads": (0, cfg["n_heads"]), "kv_heads": (0, cfg["n_kv_heads"]), "ffn": (0, cfg["ffn"]),
                "vocab": (0, cfg["vocab"])}
    if cfg["n_kv_heads"] % world or cfg["ffn"] % (32 * world) or cfg["n_heads"] % world:
        raise ValueError(f"model does not split over {world} ranks")
    h, kv, f = cfg["n_heads"] // world, cfg["n_kv_heads"] // world, cfg["ffn"] // world
    per = -(-cfg["vocab"] // (world * 16)) * 16
    v0 = min(cfg["vocab"], rank * per)
    v1 = min(cfg["vocab"], v0 + per)
    return {"heads": (rank * h, rank * h + h), "kv_heads": (rank * kv, rank * kv + kv),
            "ffn": (rank * f, rank * f + f), "vocab": (v0, v1)}


def exchange_handles(handle: bytes, group=None) -> list[bytes]:
    """All ranks' handles in rank order (an all_gather of 64-byte blobs)."""
    import torch.distributed as dist
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, handle, group=group)
    return out


def create_model(cfg: dict, group=None, safetensors: str | None = None):
    """Create this rank's shard of `cfg` (random init, or read from a safetensors
    checkpoint) and connect it to the other ranks."""
    import torch.distributed as dist
    from .engine import Model
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    m = Model(dict(cfg, tp_rank=rank, tp_size=world), safetensors=safetensors)
    if world > 1:
        m.tp_connect(exchange_handles(m.tp_handle(), group))
    return m


def create_batch(model, rows: int, group=None):
    """The batched engine over this rank's shard, connected to the other ranks."""
    import torch.distributed as dist
    from .engine import Batch
    b = Batch(model, rows)
    if dist.get_world_size(group) > 1:
        b.tp_connect(exchange_handles(b.tp_handle(), group))
    return b
