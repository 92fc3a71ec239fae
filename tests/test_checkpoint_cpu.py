"""Checkpoint loading without vLLM (minicpm5_mk.checkpoint): a Hugging Face directory round-trips into the
config and HF-named state dict that prepare_mk_weights takes."""
import pytest
import torch

from ckpt_util import write_checkpoint
from minicpm5_mk import checkpoint, mk_weights
from minicpm5_mk.mk_config import PRESETS
from minicpm5_mk.mk_init import random_state_dict


def test_checkpoint_round_trip(tmp_path):
    cfg = PRESETS["tiny-hd128"]
    sd = random_state_dict(cfg, seed=7)
    write_checkpoint(str(tmp_path), cfg, sd)
    cfg2, sd2 = checkpoint.load_hf_checkpoint(str(tmp_path), max_seq=cfg.max_seq)
    assert cfg2 == cfg
    assert set(sd) <= set(sd2)
    for k, v in sd.items():
        assert torch.equal(v, sd2[k]), k
    pw = mk_weights.prepare_mk_weights(sd2, cfg2)
    assert pw["w_qkv"].dtype == torch.int8 and pw["w_qkv"].shape[0] == cfg.num_layers


def test_tied_embeddings_and_missing_files(tmp_path):
    cfg = PRESETS["tiny-hd128"].replace(tie_embeddings=True)
    sd = random_state_dict(cfg, seed=7)
    sd.pop("lm_head.weight", None)
    write_checkpoint(str(tmp_path / "tied"), cfg, sd)
    _, sd2 = checkpoint.load_hf_checkpoint(str(tmp_path / "tied"))
    assert torch.equal(sd2["lm_head.weight"], sd2["model.embed_tokens.weight"])
    with pytest.raises(FileNotFoundError):
        checkpoint.load_hf_checkpoint(str(tmp_path / "nothing"))
