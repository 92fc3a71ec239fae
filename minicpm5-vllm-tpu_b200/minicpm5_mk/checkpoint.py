"""Real-checkpoint loading and the gate dump, outside vLLM.

* `load_hf_checkpoint(path)`: a Hugging Face checkpoint directory (`config.json` + `*.safetensors`) ->
  (MkConfig, HF-named state dict).  The reference reads these checkpoints through vLLM
  (`plugin/minicpm5_mk/model.py:599-698`) and its golden through `snapshot_download`
  (`benchmark/f32_golden.py:111-122`); this is the same data without either, so a supplied checkpoint
  can be scored offline.
* `gate_results(engine, sets, k)`: the last-position top-k log-probs of each gate set, in the layout of the
  reference's gate dumps (`run_gate`, `benchmark/run_benchmark.py:482-506`: per set
  {batch_size, seq_len, seqs: [{sampled, sampled_nolp, top_ids, top_logprobs}]}), so they can be scored
  against `benchmark/ref/*.json` with the reference's `compare_gate`.
"""

from __future__ import annotations

import glob
import json
import os
from types import SimpleNamespace
from typing import Dict, List, Tuple

import torch

from .mk_config import MkConfig, from_hf_config, rope_support


def load_hf_checkpoint(path: str, device: str | torch.device = "cpu",
                       max_seq: int = 8192) -> Tuple[MkConfig, Dict[str, torch.Tensor]]:
    """(config, state dict) of the checkpoint directory `path`.  Tensors keep their stored dtype; they are
    read onto `device` (a CUDA device makes `prepare_mk_weights` run on the GPU).  rope_theta is read from
    `rope_parameters` / `rope_scaling` where the config keeps it there; a rope type other than plain RoPE
    (yarn, longrope, ...) raises ValueError, as the vLLM model class disables its fast path for it."""
    cfg_path = os.path.join(path, "config.json")
    if not os.path.exists(cfg_path):
        raise FileNotFoundError(f"minicpm5_mk: no config.json in {path}")
    hf = SimpleNamespace(**json.load(open(cfg_path)))
    _, rope_problem = rope_support(hf)
    if rope_problem:  # the kernels apply plain RoPE only; scoring with it would be silently wrong
        raise ValueError(f"minicpm5_mk: {path}: {rope_problem}")
    cfg = from_hf_config(hf, max_seq=max_seq)
    files = sorted(glob.glob(os.path.join(path, "*.safetensors")))
    if not files:
        raise FileNotFoundError(f"minicpm5_mk: no *.safetensors in {path}")
    from safetensors.torch import load_file

    sd: Dict[str, torch.Tensor] = {}
    for f in files:
        sd.update(load_file(f, device=str(device)))
    if cfg.tie_embeddings or "lm_head.weight" not in sd:
        sd.setdefault("lm_head.weight", sd["model.embed_tokens.weight"])
    return cfg, sd


def gate_results(engine, sets: List[dict], k: int = 20) -> List[dict]:
    """Top-k dumps of `sets` (each {batch_size, seq_len, prompt_token_ids}) through `engine`
    (minicpm5_mk.ops.MkEngine): one forward per set with the logits, GPU log-softmax top-k on them.
    `sampled` is the forward's greedy token, `sampled_nolp` the greedy token of a second forward without
    logits (the scoring fast path), as the reference records both."""
    from . import ops

    out = []
    for s in sets:
        bs, seq = int(s["batch_size"]), int(s["seq_len"])
        ids = torch.tensor(s["prompt_token_ids"], dtype=torch.int32)
        if tuple(ids.shape) != (bs, seq):
            raise ValueError(f"minicpm5_mk: gate set ids {tuple(ids.shape)} != ({bs}, {seq})")
        ids = ids.reshape(-1).contiguous().to(engine.device)
        _, lg, top1 = engine.forward(ids, bs, seq, hidden=False)
        tid, tlp = ops.topk_logprobs(lg, k)
        _, _, top1_nolp = engine.forward(ids, bs, seq, hidden=False, logits=False)
        tid, tlp, top1, top1_nolp = tid.cpu(), tlp.cpu(), top1.cpu(), top1_nolp.cpu()
        seqs = [{"sampled": int(top1[b]), "sampled_nolp": int(top1_nolp[b]), "top_ids": tid[b].tolist(),
                 "top_logprobs": [round(float(v), 6) for v in tlp[b]]} for b in range(bs)]
        out.append({"batch_size": bs, "seq_len": seq, "seqs": seqs})
    return out
