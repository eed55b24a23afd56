#!/usr/bin/env python3
"""Regenerate tests/golden/tiny_weights.bin and tiny_weights.json.

Runs the reference's own exporter, python/export_weights.py:20-135
(``export_model_weights``, unmodified), on a seeded random-init SmolLM3 model
of a tiny geometry (vocab 128, hidden 128, 2 layers, 4 query / 2 KV heads of
32, intermediate 96), saved to a temporary directory first, and the
reference's fixture generator, python/reference.py:40-96
(``save_activations``, unmodified), on the same model and 40 seeded tokens;
its layer-0 dumps on the attention path (q/k/v projections, rotated q/k,
attention output, o_proj output) go to tests/golden/tiny/. The tokenizer the
exporter serialises is replaced by a stub whose JSON is a short fixed string
(the real tokenizer needs the hub), and from_pretrained is called without
device_map (accelerate is not installed). tiny_weights.json records the header
values, the tokenizer bytes and, per exported tensor, its shape and float64
sum / sum of squares / first values, taken from the model's state dict, so the
loader tests can check every tensor it carves.

    REFERENCE_ROOT=<reference checkout> python tests/golden/make_weights_fixture.py

CPU only; nothing on a GPU box runs it.
"""
from __future__ import annotations

import json
import os
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
TOKENIZER_JSON = '{"version": "stub", "model": {"type": "WordLevel", "vocab": {"a": 0}}}'


class _InnerTok:
    def to_str(self):
        return TOKENIZER_JSON


class _TokStub:
    _tokenizer = _InnerTok()


class _TokStub2:
    """save_activations only decodes the greedy token."""

    def decode(self, ids):
        return " ".join(str(i) for i in ids)


def main() -> None:
    if "REFERENCE_ROOT" not in os.environ:
        raise SystemExit("set REFERENCE_ROOT to the reference checkout (the directory holding python/)")
    sys.path.insert(0, str(Path(os.environ["REFERENCE_ROOT"]) / "python"))
    import numpy as np
    import torch
    from transformers import SmolLM3Config, SmolLM3ForCausalLM

    import export_weights  # python/export_weights.py of the reference checkout
    from model_config import ModelConfig

    torch.manual_seed(77)
    cfg = SmolLM3Config(vocab_size=128, hidden_size=128, intermediate_size=96, num_hidden_layers=2,
                        num_attention_heads=4, num_key_value_heads=2, head_dim=32, max_position_embeddings=512,
                        initializer_range=0.1, rope_parameters={"rope_type": "default", "rope_theta": 5.0e6},
                        tie_word_embeddings=True, pad_token_id=0, bos_token_id=1, eos_token_id=2)
    model = SmolLM3ForCausalLM(cfg).eval()
    with torch.no_grad():   # norms away from 1.0 so a swapped tensor shows
        for n, p in model.named_parameters():
            if "norm" in n:
                p.copy_(torch.rand_like(p) + 0.5)
    with tempfile.TemporaryDirectory() as tmp:
        model.save_pretrained(tmp)
        export_weights.get_tokenizer = lambda _path: _TokStub()
        # accelerate (needed by from_pretrained's device_map="cpu") is not in
        # this image: load the saved model the same way without that argument
        real = export_weights.AutoModelForCausalLM

        class _Loader:
            @staticmethod
            def from_pretrained(path, **kw):
                kw.pop("device_map", None)
                kw.pop("low_cpu_mem_usage", None)
                return real.from_pretrained(path, **kw)
        export_weights.AutoModelForCausalLM = _Loader
        mc = ModelConfig(cfg)
        out = HERE / "tiny_weights.bin"
        export_weights.export_model_weights(mc, tmp, out)
    # the fixture generator on the same model (fp16, as from_pretrained gives it)
    import reference  # python/reference.py of the reference checkout
    tiny = HERE / "tiny"
    tiny.mkdir(exist_ok=True)
    m16 = model.to(torch.float16).eval()
    ids = torch.randint(0, cfg.vocab_size, (1, 40), generator=torch.Generator().manual_seed(78))
    with tempfile.TemporaryDirectory() as tmp:
        reference.save_activations(m16, _TokStub2(), Path(tmp), 40, ids)
        for name in ("layer0_q_proj_out", "layer0_k_proj_out", "layer0_v_proj_out", "layer0_q_rope",
                     "layer0_k_rope", "layer0_attn_out", "layer0_o_proj_out"):
            (tiny / f"{name}.bin").write_bytes((Path(tmp) / f"{name}.bin").read_bytes())
    sd = {k: v.to(torch.float16).float().numpy().astype(np.float64) for k, v in model.state_dict().items()}
    order = ["model.embed_tokens.weight"]
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        order += [p + "input_layernorm.weight", p + "self_attn.q_proj.weight", p + "self_attn.k_proj.weight",
                  p + "self_attn.v_proj.weight", p + "self_attn.o_proj.weight",
                  p + "post_attention_layernorm.weight", p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight",
                  p + "mlp.down_proj.weight"]
    order += ["model.norm.weight", "model.embed_tokens.weight"]   # lm_head: tied, written again
    tensors = [{"name": n if j < len(order) - 1 else "lm_head.weight (tied)", "shape": list(sd[n].shape),
                "sum": float(sd[n].sum()), "sumsq": float((sd[n] ** 2).sum()),
                "first": [float(x) for x in sd[n].reshape(-1)[:4]]} for j, n in enumerate(order)]
    meta = {"generator": "python/export_weights.py export_model_weights (reference checkout, unmodified), "
                         "random-init tiny SmolLM3 (seed 77), stub tokenizer",
            "header": {"vocab_size": mc.vocab_size, "hidden_size": mc.hidden_size, "num_layers": mc.num_layers,
                       "num_heads": mc.num_heads, "num_kv_heads": mc.num_kv_heads, "head_dim": mc.head_dim,
                       "intermediate_size": mc.intermediate_size, "max_seq_len": mc.max_seq_len,
                       "rms_norm_eps": mc.rms_norm_eps, "rope_theta": mc.rope_theta},
            "tokenizer_json": TOKENIZER_JSON, "tensors": tensors}
    (HERE / "tiny_weights.json").write_text(json.dumps(meta, indent=1) + "\n")
    print(f"wrote {out.name} ({out.stat().st_size} bytes) and tiny_weights.json")


if __name__ == "__main__":
    main()
