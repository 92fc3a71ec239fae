"""Child process of tests/test_vllm_drop_in_gpu.py (one vLLM engine per process).

    python tests/vllm_drop_in_child.py make <dir>    # tiny Llama-format checkpoint + prompts + golden top-1
    python tests/vllm_drop_in_child.py mk <dir>      # LLM.generate through MiniCPM5MegakernelForCausalLM
    python tests/vllm_drop_in_child.py stock <dir>   # same, MINICPM5_MK_ENABLE=0 (vLLM's own Llama path)
    python tests/vllm_drop_in_child.py mkfree <dir>  # plugin path with MINICPM5_MK_FREE_STOCK=1 (KV-cache skip)

Prints one JSON line.  The checkpoint is the tiny-hd96 preset with plain-Llama scalars (the muP
scalars at 1.0, so vLLM's stock Llama and the megakernel compute the same model), random weights
N(0, 0.02) from seed 1234 stored in bf16, and 4 prompts of 256 ids."""
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(ROOT, "minicpm5-vllm-tpu_b200"))
sys.path.insert(0, ROOT)


def make(mdir):
    import torch
    from safetensors.torch import save_file
    from minicpm5_mk.mk_config import PRESETS
    from minicpm5_mk.mk_init import random_state_dict, synthetic_ids
    from oracle import golden

    cfg = PRESETS["tiny-hd96"].replace(scale_emb=1.0, residual_scale=1.0, logit_scale=1.0, max_seq=1024)
    sd = {k: v.to(torch.bfloat16) for k, v in random_state_dict(cfg, seed=1234).items()}
    os.makedirs(mdir, exist_ok=True)
    save_file({k: v.contiguous() for k, v in sd.items()}, os.path.join(mdir, "model.safetensors"))
    hf = {"architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": cfg.hidden,
          "intermediate_size": cfg.inter, "num_hidden_layers": cfg.num_layers, "num_attention_heads": cfg.n_q,
          "num_key_value_heads": cfg.n_kv, "head_dim": cfg.head_dim, "vocab_size": cfg.vocab,
          "max_position_embeddings": 1024, "rms_norm_eps": cfg.eps, "rope_theta": cfg.rope_theta,
          "tie_word_embeddings": False, "torch_dtype": "bfloat16", "hidden_act": "silu",
          "bos_token_id": 1, "eos_token_id": 2}
    with open(os.path.join(mdir, "config.json"), "w") as f:
        json.dump(hf, f)
    ids = synthetic_ids(4, 256, seed=7, vocab=cfg.vocab)
    W = golden.golden_weights({k: v.float() for k, v in sd.items()}, cfg)
    top1 = [golden.argmax_first(golden.forward_logits(ids[b], W, cfg)) for b in range(ids.shape[0])]
    with open(os.path.join(mdir, "prompts.json"), "w") as f:
        json.dump({"ids": ids.tolist(), "golden_top1": top1}, f)
    print(json.dumps({"made": mdir, "golden_top1": top1}))


def generate(mdir, fast, free_stock=False):
    if fast:
        os.environ["MINICPM5_MK_STATUS_DIR"] = os.path.join(mdir, "status")
        if free_stock:  # no stock fallback: the KV-cache allocation skip applies
            os.environ["MINICPM5_MK_FREE_STOCK"] = "1"
    else:
        os.environ["MINICPM5_MK_ENABLE"] = "0"
    from vllm import LLM, SamplingParams

    p = json.load(open(os.path.join(mdir, "prompts.json")))
    llm = LLM(model=mdir, skip_tokenizer_init=True, hf_overrides={"architectures": ["MiniCPM5MegakernelForCausalLM"]},
              max_model_len=1024, enforce_eager=True, gpu_memory_utilization=0.3, max_num_batched_tokens=2048,
              max_num_seqs=8, dtype="bfloat16")
    outs = llm.generate([{"prompt_token_ids": x} for x in p["ids"]],
                        SamplingParams(max_tokens=1, temperature=0.0, detokenize=False))
    status = None
    sp = os.path.join(mdir, "status", "minicpm5_mk_status_rank0.json")
    if fast and os.path.exists(sp):
        status = json.load(open(sp))
    print(json.dumps({"tokens": [o.outputs[0].token_ids[0] for o in outs], "status": status}))


if __name__ == "__main__":
    what, mdir = sys.argv[1], sys.argv[2]
    if what == "make":
        make(mdir)
    else:
        generate(mdir, what in ("mk", "mkfree"), free_stock=what == "mkfree")
