"""Write a model as a Hugging Face checkpoint directory (config.json + model.safetensors), as the
checkpoint-loading tests need one."""
import json
import os


def write_checkpoint(path, cfg, sd):
    from safetensors.torch import save_file
    os.makedirs(path, exist_ok=True)
    hf = {"architectures": ["LlamaForCausalLM"], "model_type": "llama", "num_hidden_layers": cfg.num_layers,
          "hidden_size": cfg.hidden, "intermediate_size": cfg.inter, "num_attention_heads": cfg.n_q,
          "num_key_value_heads": cfg.n_kv, "head_dim": cfg.head_dim, "vocab_size": cfg.vocab,
          "rope_theta": cfg.rope_theta, "rms_norm_eps": cfg.eps, "tie_word_embeddings": cfg.tie_embeddings,
          "torch_dtype": "float32"}
    json.dump(hf, open(os.path.join(path, "config.json"), "w"))
    save_file({k: v.contiguous() for k, v in sd.items()}, os.path.join(path, "model.safetensors"))
