"""Write a synthetic Qwen2-1.5B-attention-shaped .qwn model for the qwnrun
drop-in tests (TEST INFRASTRUCTURE ONLY, run where the reference checkout
is present; the file lands in oracle/_ref and travels to the GPU box).

Shapes: 2 layers, 12 query heads, 2 KV heads, head_dim 128 (the cfg1
attention shapes), hidden size 256, MLP 256, vocabulary 64, weights from a
seeded generator.  Two variants of the same weights:

* f32 projections: the CPU decoder runs them in fp32, so logits move
  smoothly with the KV-cache path alone (the relinked-decoder checks);
* --hvsq2: every projection and the LM head in HyperVSQ-2 (74-byte blocks
  of 256 weights), since qwnrun's CUDA backend runs only those on the GPU
  (c/qwanto_decode.c:783-870); their int8 activations re-round at every
  projection, so tiny upstream differences move logits in steps.

Embeddings and norms stay f32.  The container and the quantized blocks are
written by the reference's own converter, c/tools/qwn_convert.py (write_qwn,
quantize_hyper_vsq2_rows), the way c/tests/test_qwn_decoder.py:26-55 builds
its fixture.

    python oracle/make_qwn_fixture.py OUT.qwn [--hvsq2]
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

HIDDEN, INTER, LAYERS, HEADS, KV_HEADS, HEAD_DIM, VOCAB, MAX_POS = 256, 256, 2, 12, 2, 128, 64, 2048


def main(out: str, hvsq2: bool) -> int:
    from refpath import reference_c
    ref = reference_c()
    if ref is None:
        print("reference checkout not found; fixture not written", file=sys.stderr)
        return 1
    sys.path.insert(0, ref)
    from tools.qwn_convert import DT_BYTES, DT_F32, DT_HYPER_VSQ2, quantize_hyper_vsq2_rows, write_qwn

    rng = np.random.default_rng(20260)

    def mat(rows, cols, std):  # payload row-major [rows][cols]; .qwn shape lists the fastest dim first
        w = (rng.standard_normal((rows, cols)) * std).astype("<f4")
        return {"dtype": DT_F32, "shape": (cols, rows), "payload": w.tobytes()}

    def hvsq(rows, cols, std):
        w = (rng.standard_normal((rows, cols)) * std).astype("<f4")
        if not hvsq2:
            return {"dtype": DT_F32, "shape": (cols, rows), "payload": w.tobytes()}
        return {"dtype": DT_HYPER_VSQ2, "shape": (cols, rows),
                "payload": quantize_hyper_vsq2_rows(w.tobytes(), rows, cols)}

    def vec(n, center=1.0, spread=0.05):
        v = (center + rng.standard_normal(n) * spread).astype("<f4")
        return {"dtype": DT_F32, "shape": (n,), "payload": v.tobytes()}

    cfg = {"hidden_size": HIDDEN, "intermediate_size": INTER, "num_hidden_layers": LAYERS,
           "num_attention_heads": HEADS, "num_key_value_heads": KV_HEADS, "head_dim": HEAD_DIM,
           "vocab_size": VOCAB, "max_position_embeddings": MAX_POS, "rms_norm_eps": 1e-6,
           "rope_theta": 1000000.0, "bos_token_id": -1, "eos_token_id": VOCAB - 1,
           "tie_word_embeddings": False}
    tok = {"model": {"type": "BPE", "vocab": {chr(48 + i): i for i in range(VOCAB)}, "merges": []},
           "added_tokens": []}
    cfg_b, tok_b = json.dumps(cfg).encode(), json.dumps(tok).encode()
    tensors = [{"name": "__qwn.config", "dtype": DT_BYTES, "shape": (len(cfg_b),), "payload": cfg_b},
               {"name": "__qwn.tokenizer", "dtype": DT_BYTES, "shape": (len(tok_b),), "payload": tok_b},
               dict(name="model.embed_tokens.weight", **mat(VOCAB, HIDDEN, 1.0))]
    for l in range(LAYERS):
        p = f"model.layers.{l}."
        tensors += [dict(name=p + "input_layernorm.weight", **vec(HIDDEN)),
                    dict(name=p + "self_attn.q_proj.weight", **hvsq(HEADS * HEAD_DIM, HIDDEN, 0.08)),
                    dict(name=p + "self_attn.k_proj.weight", **hvsq(KV_HEADS * HEAD_DIM, HIDDEN, 0.08)),
                    dict(name=p + "self_attn.v_proj.weight", **hvsq(KV_HEADS * HEAD_DIM, HIDDEN, 0.08)),
                    dict(name=p + "self_attn.o_proj.weight", **hvsq(HIDDEN, HEADS * HEAD_DIM, 0.02)),
                    dict(name=p + "post_attention_layernorm.weight", **vec(HIDDEN)),
                    dict(name=p + "mlp.gate_proj.weight", **hvsq(INTER, HIDDEN, 0.06)),
                    dict(name=p + "mlp.up_proj.weight", **hvsq(INTER, HIDDEN, 0.06)),
                    dict(name=p + "mlp.down_proj.weight", **hvsq(HIDDEN, INTER, 0.12))]
    tensors += [dict(name="model.norm.weight", **vec(HIDDEN)),
                dict(name="lm_head.weight", **hvsq(VOCAB, HIDDEN, 0.1))]
    write_qwn(out, tensors, arch_dims=(HIDDEN, INTER, HEADS, KV_HEADS, HEAD_DIM, LAYERS, VOCAB, MAX_POS))
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1], "--hvsq2" in sys.argv[2:]))
