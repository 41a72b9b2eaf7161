"""Head-sharded tensor parallelism for the packed refresh (70B-class models).

The reference runs on one device (api.py:156-160, kernels/packed_cache.py:
145-151). For models whose weights do not fit one GPU, each of P ranks (one
process per GPU) holds:

* q/k/v rows of its Hq/P query heads and Hkv/P KV heads (column-parallel),
* the matching columns of o_proj (row-parallel),
* 1/P of the MLP: gate/up rows (column-parallel) and down columns (row-parallel),
* the norms and the embedding in full, and
* its KV heads' slice of the cache.

Per layer the two row-parallel projections produce partial sums that NCCL
all-reduces in place (sum) before the residual add; everything else (RoPE
fix, K/V scatter, attention) is local to the rank's heads. With P = 1 this is
the single-GPU engine.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .engine import LayerWeights, refresh_rows

SHARDED_NAMES = ("q", "k", "v", "o", "gate", "up", "down")
REPLICATED_NAMES = ("in_norm", "post_norm", "q_norm", "k_norm")


def shard_range(total: int, rank: int, world: int) -> slice:
    if total % world:
        raise ValueError(f"{total} is not divisible by the tensor-parallel degree {world}")
    part = total // world
    return slice(rank * part, (rank + 1) * part)


def shard_layer_tensors(layer: dict, *, heads: int, kv_heads: int, head_dim: int, intermediate: int,
                        rank: int, world: int) -> dict:
    """This rank's share of one decoder layer, given full weights by name
    (``q k v o gate up down`` as nn.Linear ``[out, in]``, norms as vectors)."""
    qs = shard_range(heads, rank, world)
    ks = shard_range(kv_heads, rank, world)
    ms = shard_range(intermediate, rank, world)
    rows_q = slice(qs.start * head_dim, qs.stop * head_dim)
    rows_kv = slice(ks.start * head_dim, ks.stop * head_dim)
    out = {
        "q": layer["q"][rows_q].contiguous(),
        "k": layer["k"][rows_kv].contiguous(),
        "v": layer["v"][rows_kv].contiguous(),
        "o": layer["o"][:, rows_q].contiguous(),
        "gate": layer["gate"][ms].contiguous(),
        "up": layer["up"][ms].contiguous(),
        "down": layer["down"][:, ms].contiguous(),
    }
    for name in REPLICATED_NAMES:
        if layer.get(name) is not None:
            out[name] = layer[name]
    return out


def kv_head_shard(cache_tensor: torch.Tensor, kv_heads: int, rank: int, world: int) -> torch.Tensor:
    """This rank's KV heads of a ``[1, Hkv, N, D]`` cache tensor (a view)."""
    return cache_tensor[:, shard_range(kv_heads, rank, world)]


def rope_tables(inv_freq: torch.Tensor, positions: torch.Tensor, dtype: torch.dtype, attention_scaling: float = 1.0):
    """cos/sin ``[B, D]`` by the rotary forward's own op sequence (transformers
    LlamaRotaryEmbedding.forward): ``inv_freq @ positions`` in fp32 (K=1),
    duplicated halves, cos/sin, scaling, cast to the model dtype."""
    inv = inv_freq.to(positions.device)[None, :, None].float()
    pos = positions[None, None, :].float()
    freqs = (inv @ pos).transpose(1, 2)
    emb = torch.cat((freqs, freqs), dim=-1)
    cos = emb.cos() * attention_scaling
    sin = emb.sin() * attention_scaling
    return cos[0].to(dtype).contiguous(), sin[0].to(dtype).contiguous()


class ShardView:
    """One rank's shard of a dense Llama/Qwen3 decoder, in the form
    ``engine.refresh_rows`` consumes (the same fields as ``ModelView``)."""

    def __init__(self, *, embed, layers: list[dict], hidden: int, heads: int, kv_heads: int, head_dim: int,
                 intermediate: int, eps: float, inv_freq: torch.Tensor, rank: int, world: int,
                 attention_scaling: float = 1.0):
        self.embed = embed
        self.hidden = hidden
        self.heads = heads // world
        self.kv_heads = kv_heads // world
        self.head_dim = head_dim
        self.intermediate = intermediate // world
        self.eps = float(eps)
        self.vocab = embed.shape[0]
        self.dtype = embed.dtype
        self.inv_freq = inv_freq
        self.attention_scaling = attention_scaling
        self.rank, self.world = rank, world
        self.layers = [LayerWeights(in_norm=d["in_norm"], q=d["q"], k=d["k"], v=d["v"], o=d["o"],
                                    post_norm=d["post_norm"], gate=d["gate"], up=d["up"], down=d["down"],
                                    q_norm=d.get("q_norm"), k_norm=d.get("k_norm")) for d in layers]

    @classmethod
    def from_model(cls, base, rank: int, world: int) -> "ShardView":
        """Shard a full transformers LlamaModel/Qwen3Model held by this rank."""
        config = base.config
        head_dim = getattr(config, "head_dim", None) or config.hidden_size // config.num_attention_heads
        layers = []
        for layer in base.layers:
            attn, mlp = layer.self_attn, layer.mlp
            full = {"in_norm": layer.input_layernorm.weight, "q": attn.q_proj.weight, "k": attn.k_proj.weight,
                    "v": attn.v_proj.weight, "o": attn.o_proj.weight,
                    "post_norm": layer.post_attention_layernorm.weight, "gate": mlp.gate_proj.weight,
                    "up": mlp.up_proj.weight, "down": mlp.down_proj.weight,
                    "q_norm": getattr(getattr(attn, "q_norm", None), "weight", None),
                    "k_norm": getattr(getattr(attn, "k_norm", None), "weight", None)}
            layers.append(shard_layer_tensors({k: v.detach() if v is not None else None for k, v in full.items()},
                                              heads=config.num_attention_heads,
                                              kv_heads=config.num_key_value_heads, head_dim=head_dim,
                                              intermediate=config.intermediate_size, rank=rank, world=world))
        return cls(embed=base.embed_tokens.weight.detach(), layers=layers, hidden=config.hidden_size,
                   heads=config.num_attention_heads, kv_heads=config.num_key_value_heads, head_dim=head_dim,
                   intermediate=config.intermediate_size, eps=config.rms_norm_eps, inv_freq=base.rotary_emb.inv_freq,
                   rank=rank, world=world, attention_scaling=getattr(base.rotary_emb, "attention_scaling", 1.0))

    def rope_tables(self, positions: torch.Tensor):
        return rope_tables(self.inv_freq, positions, self.dtype, self.attention_scaling)


class TPGroup:
    """An NCCL communicator over the ranks of a torch.distributed group, for
    the in-loop all-reduces of ``kvr_packed_refresh``."""

    def __init__(self, rank: int, world: int, device: torch.device, group=None):
        import torch.distributed as dist

        lib = _lib.load()
        ident = torch.zeros(_lib.TP_ID_BYTES, dtype=torch.uint8)
        if rank == 0:
            buf = (ctypes.c_uint8 * _lib.TP_ID_BYTES)()
            _lib.check(lib.kvr_tp_unique_id(ctypes.cast(buf, ctypes.c_void_p)), "tp_unique_id")
            ident = torch.tensor(list(bytes(buf)), dtype=torch.uint8)
        backend = dist.get_backend(group)
        carrier = ident.to(device) if backend == "nccl" else ident
        dist.broadcast(carrier, src=0, group=group)
        ident = carrier.cpu()
        raw = (ctypes.c_uint8 * _lib.TP_ID_BYTES)(*ident.tolist())
        comm = ctypes.c_void_p()
        with torch.cuda.device(device):
            _lib.check(lib.kvr_tp_comm_init(ctypes.cast(raw, ctypes.c_void_p), world, rank, ctypes.byref(comm)),
                       "tp_comm_init")
        self.comm = comm.value
        self.rank, self.world, self.device = rank, world, device

    def close(self):
        if self.comm:
            _lib.check(_lib.load().kvr_tp_comm_destroy(self.comm), "tp_comm_destroy")
            self.comm = None


def refresh_rows_tp(view: ShardView, layers, ids, positions, max_position: int, cache_rows: int,
                    group: TPGroup, sources=None) -> None:
    """``engine.refresh_rows`` on this rank's shard; ``layers`` (and the
    optional ``sources`` they first copy) hold this rank's KV heads. Every rank
    of the group must call it with the same ids and positions."""
    refresh_rows(view, layers, ids, positions, max_position, cache_rows, tp_comm=group.comm if group else None,
                 sources=sources)
