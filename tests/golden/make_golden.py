#!/usr/bin/env python3
"""Regenerate the golden vectors in this directory.

The reference engine's own fixtures (tests/reference/*.bin) come from its
fixture generator, python/reference.py:40-96 (``save_activations``), run on
the HF SmolLM3-3B checkpoint; neither the fixtures nor the checkpoint are
available. This script runs that same, unmodified ``save_activations`` on a
seeded random-init SmolLM3 model of the same attention geometry (16 query
heads, 4 KV heads, head_dim 128, RoPE theta 5e6, FP16 on CPU) and keeps the
dumps on the attention hot path:

    layer0_q_proj_out.bin  layer0_k_proj_out.bin  layer0_v_proj_out.bin
    layer0_q_rope.bin      layer0_k_rope.bin      layer0_attn_out.bin

Each is raw little-endian FP16 exactly as python/reference.py:18-22 writes
it. ``meta.json`` records the geometry, seed and library versions.

It needs the reference checkout (set REFERENCE_ROOT to the directory that
holds python/reference.py) and runs on CPU only. Nothing on a GPU box runs
it; the tests read only the committed outputs.

Two sets are committed:

    REFERENCE_ROOT=... python tests/golden/make_golden.py
        40 tokens, seed 1234, initializer_range 0.04 (this directory);
    REFERENCE_ROOT=... python tests/golden/make_golden.py --seq-len 160 \
        --seed 4321 --init-range 0.08 --out tests/golden/sharp
        160 tokens (across the 128-token tile edge), larger weights: the
        attention logits have a standard deviation of about 13 instead of
        about 3, so the softmax is peaked and the fixture pins its max and
        normalisation, not only RoPE and the layout.
"""
from __future__ import annotations

import json
import os
import shutil
import sys
import tempfile
from pathlib import Path

KEEP = ["layer0_q_proj_out", "layer0_k_proj_out", "layer0_v_proj_out",
        "layer0_q_rope", "layer0_k_rope", "layer0_attn_out"]


class _TokenizerStub:
    """save_activations only calls tokenizer.decode on the greedy token."""

    def decode(self, ids):
        return " ".join(str(i) for i in ids)


def main(seq_len: int = 40, seed: int = 1234, out_dir: str | None = None, init_range: float = 0.04) -> None:
    if "REFERENCE_ROOT" not in os.environ:
        raise SystemExit("set REFERENCE_ROOT to the reference checkout (the directory holding python/reference.py)")
    ref_root = Path(os.environ["REFERENCE_ROOT"])
    sys.path.insert(0, str(ref_root / "python"))
    import torch
    import transformers
    from transformers import SmolLM3Config, SmolLM3ForCausalLM

    import reference  # python/reference.py of the reference checkout

    torch.manual_seed(seed)
    config = SmolLM3Config(
        vocab_size=1024, hidden_size=2048, intermediate_size=512,
        num_hidden_layers=1, num_attention_heads=16, num_key_value_heads=4,
        max_position_embeddings=4096, initializer_range=init_range,
        rope_parameters={"rope_type": "default", "rope_theta": 5.0e6},
        tie_word_embeddings=True, pad_token_id=0, bos_token_id=1, eos_token_id=2,
    )
    # _from_config(dtype=fp16) builds the model the way from_pretrained(
    # torch_dtype=fp16) does (python/reference.py:137-143): weights in FP16,
    # the rotary inv_freq buffer left in FP32.
    model = SmolLM3ForCausalLM._from_config(config, dtype=torch.float16).eval()
    assert model.model.rotary_emb.inv_freq.dtype == torch.float32
    gen = torch.Generator().manual_seed(seed + 1)
    input_ids = torch.randint(0, config.vocab_size, (1, seq_len), generator=gen)

    out = Path(out_dir) if out_dir else Path(__file__).resolve().parent
    out.mkdir(parents=True, exist_ok=True)
    with tempfile.TemporaryDirectory() as tmp:
        reference.save_activations(model, _TokenizerStub(), Path(tmp), seq_len, input_ids)
        for name in KEEP:
            shutil.copyfile(Path(tmp) / f"{name}.bin", out / f"{name}.bin")
    meta = {
        "generator": "python/reference.py save_activations (reference checkout, unmodified)",
        "model": f"SmolLM3ForCausalLM, random init (initializer_range {init_range}), 1 layer, fp16, CPU",
        "seq_len": seq_len, "num_heads": 16, "num_kv_heads": 4, "head_dim": 128,
        "rope_theta": 5.0e6, "seed": seed,
        "torch": torch.__version__, "transformers": transformers.__version__,
        "reference_pins": {"torch": "2.14.0+rocm (python/requirements.txt:79)",
                           "transformers": "5.17.0 (python/requirements.txt:82)"},
        "files": {name: f"{name}.bin" for name in KEEP},
    }
    (out / "meta.json").write_text(json.dumps(meta, indent=2) + "\n")
    print(f"wrote {len(KEEP)} fixtures to {out}")


if __name__ == "__main__":
    import argparse
    ap = argparse.ArgumentParser()
    ap.add_argument("--seq-len", type=int, default=40)
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--init-range", type=float, default=0.04)
    ap.add_argument("--out", default=None)
    args = ap.parse_args()
    main(args.seq_len, args.seed, args.out, args.init_range)
