"""weights.bin reader (Python mirror of include/b200attn/weights.hpp).

The format the reference's python/export_weights.py:20-135 writes and its
include/model.hpp:17-92 / include/device_weights.hpp:56-108 read: a 44-byte
header ("QWEN", 8 x uint32, 2 x float32), a uint32 tokenizer JSON length and
the JSON, zero padding to a 64-byte offset, then FP16 tensors in network
order. ``read_weights`` maps the file, checks the header and the payload size
and returns numpy views of every tensor under the reference's field names;
``upload`` puts the whole payload on a device as one tensor (one copy) and
returns device views in the same layout.
"""
from __future__ import annotations

import dataclasses
import struct

import numpy as np

HEADER = struct.Struct("<4sIIIIIIIIff")
assert HEADER.size == 44

BLOCK_FIELDS = ("input_normalization", "q_proj", "k_proj", "v_proj", "o_proj", "post_attn_norm", "gate_proj",
                "up_proj", "down_proj")


@dataclasses.dataclass(frozen=True)
class ModelConfig:
    vocab_size: int
    hidden_size: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate_size: int
    max_seq_len: int
    rms_norm_eps: float
    rope_theta: float


def parse_header(buf) -> ModelConfig:
    if len(buf) < HEADER.size:
        raise ValueError("weights.bin: shorter than its 44-byte header")
    magic, *rest = HEADER.unpack_from(buf, 0)
    if magic != b"QWEN":
        raise ValueError("weights.bin: magic is not 'QWEN'")
    return ModelConfig(*rest)


def weights_offset(tokenizer_bytes: int) -> int:
    """include/model.hpp:72-76: header + length word + JSON, rounded up to 64."""
    return (HEADER.size + 4 + tokenizer_bytes + 63) & ~63


def layout(c: ModelConfig) -> list[tuple[str, tuple[int, ...]]]:
    """(name, shape) of every tensor in file order (device_weights.hpp:74-108)."""
    h, q, kv, inter = c.hidden_size, c.num_heads * c.head_dim, c.num_kv_heads * c.head_dim, c.intermediate_size
    shapes = {"input_normalization": (h,), "q_proj": (q, h), "k_proj": (kv, h), "v_proj": (kv, h),
              "o_proj": (h, q), "post_attn_norm": (h,), "gate_proj": (inter, h), "up_proj": (inter, h),
              "down_proj": (h, inter)}
    out = [("embedding_tokens", (c.vocab_size, h))]
    for i in range(c.num_layers):
        out += [(f"layers.{i}.{f}", shapes[f]) for f in BLOCK_FIELDS]
    out += [("final_norm", (h,)), ("lm_head", (c.vocab_size, h))]
    return out


@dataclasses.dataclass
class HostWeights:
    config: ModelConfig
    tokenizer_json: bytes
    payload: np.ndarray              # all weights, fp16, file order
    tensors: dict[str, np.ndarray]   # views into payload


def read_weights(path: str) -> HostWeights:
    raw = np.memmap(path, dtype=np.uint8, mode="r")
    cfg = parse_header(raw[:HEADER.size].tobytes())
    if raw.size < HEADER.size + 4:
        raise ValueError("weights.bin: missing the tokenizer length field")
    tok_len = int(np.frombuffer(raw[HEADER.size:HEADER.size + 4].tobytes(), "<u4")[0])
    if raw.size < HEADER.size + 4 + tok_len:
        raise ValueError("weights.bin: tokenizer payload truncated")
    tok = raw[HEADER.size + 4:HEADER.size + 4 + tok_len].tobytes()
    off = weights_offset(tok_len)
    lay = layout(cfg)
    need = sum(int(np.prod(s)) for _, s in lay) * 2
    have = raw.size - off
    if have != need:
        raise ValueError(f"weights.bin: payload is {max(have, 0)} bytes, the header implies {need} "
                         "(a file with q_norm / k_norm tensors is not this layout)")
    payload = raw[off:].view(np.float16)
    tensors, cur = {}, 0
    for name, shape in lay:
        n = int(np.prod(shape))
        tensors[name] = payload[cur:cur + n].reshape(shape)
        cur += n
    return HostWeights(cfg, tok, payload, tensors)


def upload(w: HostWeights, device):
    """One device tensor holding the payload and views of it per name."""
    import torch
    buf = torch.from_numpy(np.array(w.payload, copy=True)).to(device)
    views, cur = {}, 0
    for name, arr in w.tensors.items():
        n = arr.size
        views[name] = buf[cur:cur + n].view(arr.shape)
        cur += n
    return buf, views
