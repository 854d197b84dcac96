"""Golden logits for the decode-step integration test, from the reference's
own PFlashModelForCausalLM (polarflash_core/model_integration.py:203-254).

    POLARFLASH_REF=/path/to/POLAR-FLASH python tests/golden/make_decode_golden.py

The tiny model of tests/decode_model.py (seeded weights, oracle INT4 g128
payloads decoded back to dense W_hat) is loaded into the reference model;
it runs the prompt (prefill, causal mask) and then three single-token steps
with its KV caches.  Writes decode_step.npz: prompt, decode tokens, prefill
and step logits.  Needs the reference sources at $POLARFLASH_REF (required);
the GPU machines only read the .npz.
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("POLARFLASH_REF")
if not REF or not os.path.isdir(REF):
    sys.exit("set POLARFLASH_REF to a checkout of the reference POLAR-FLASH sources")
sys.path[:0] = [os.path.dirname(HERE), ROOT, os.path.join(ROOT, "polar-flash_b200"), REF]

import decode_model as dm  # noqa: E402
from polarflash_core.model_integration import PFlashModelForCausalLM  # noqa: E402


def main():
    w = dm.build()
    model = PFlashModelForCausalLM(dm.CFG, device="cpu")
    with torch.no_grad():
        model.embed_tokens.weight.copy_(torch.from_numpy(w["embed"]))
        model.norm.weight.copy_(torch.from_numpy(w["final_norm"]))
        model.lm_head.weight.copy_(torch.from_numpy(w["lm_head"]))
        for layer, ly in zip(model.layers, w["layers"]):
            at, mlp = layer.self_attn, layer.mlp
            at.q_weight = torch.from_numpy(ly["q"]["W_hat"])
            at.k_weight = torch.from_numpy(ly["k"]["W_hat"])
            at.v_weight = torch.from_numpy(ly["v"]["W_hat"])
            at.o_weight = torch.from_numpy(ly["o"]["W_hat"])
            mlp.gate_weight = torch.from_numpy(ly["gate"]["W_hat"])
            mlp.up_weight = torch.from_numpy(ly["up"]["W_hat"])
            mlp.down_weight = torch.from_numpy(ly["down"]["W_hat"])
            layer.input_layernorm.weight.copy_(torch.from_numpy(ly["in_norm"]))
            layer.post_attention_layernorm.weight.copy_(torch.from_numpy(ly["post_norm"]))
        caches = [{} for _ in range(dm.CFG["num_hidden_layers"])]
        pre, caches = model(torch.tensor([dm.PROMPT]), kv_caches=caches)
        steps = []
        for tok in dm.DECODE:
            lg, caches = model(torch.tensor([[tok]]), kv_caches=caches)
            steps.append(lg[0, -1].numpy())
    np.savez_compressed(os.path.join(HERE, "decode_step.npz"), prompt=np.array(dm.PROMPT), decode=np.array(dm.DECODE),
                        prefill_logits=pre[0].numpy().astype(np.float32),
                        step_logits=np.stack(steps).astype(np.float32))
    print("wrote decode_step.npz")


if __name__ == "__main__":
    main()
