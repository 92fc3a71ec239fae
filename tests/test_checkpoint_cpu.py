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


def _rewrite_config(path, **changes):
    import json
    import os
    p = os.path.join(path, "config.json")
    hf = json.load(open(p))
    for k, v in changes.items():
        if v is None:
            hf.pop(k, None)
        else:
            hf[k] = v
    json.dump(hf, open(p, "w"))


def test_rope_theta_from_rope_parameters(tmp_path):
    """A config that keeps rope_theta only inside rope_parameters (the real MiniCPM5 theta 5e6) is read
    with that theta, not the 10000 default (`plugin/minicpm5_mk/model.py:576-585`)."""
    cfg = PRESETS["tiny-hd128"]
    write_checkpoint(str(tmp_path), cfg, random_state_dict(cfg, seed=7))
    _rewrite_config(str(tmp_path), rope_theta=None, rope_parameters={"rope_theta": 5e6, "rope_type": "default"})
    cfg2, _ = checkpoint.load_hf_checkpoint(str(tmp_path), max_seq=cfg.max_seq)
    assert cfg2.rope_theta == 5e6
    assert cfg2 == cfg.replace(rope_theta=5e6)


@pytest.mark.parametrize("rope", [{"rope_type": "yarn", "factor": 4.0, "rope_theta": 5e6},
                                  {"type": "linear", "factor": 2.0}, "dynamic"])
def test_unsupported_rope_type_is_refused(tmp_path, rope):
    """Scaled RoPE variants are refused instead of being scored with plain RoPE."""
    cfg = PRESETS["tiny-hd128"]
    write_checkpoint(str(tmp_path), cfg, random_state_dict(cfg, seed=7))
    _rewrite_config(str(tmp_path), rope_scaling=rope)
    with pytest.raises(ValueError, match="unsupported"):
        checkpoint.load_hf_checkpoint(str(tmp_path), max_seq=cfg.max_seq)


def test_rope_support_helper():
    from types import SimpleNamespace
    from minicpm5_mk.mk_config import rope_support
    assert rope_support(SimpleNamespace(rope_theta=1e4)) == (None, None)
    assert rope_support(SimpleNamespace(rope_scaling={"rope_type": "default", "rope_theta": 5e6})) == (5e6, None)
    assert rope_support(SimpleNamespace(rope_scaling=None, rope_parameters={"rope_theta": 2.5e5})) == (2.5e5, None)
    theta, problem = rope_support(SimpleNamespace(rope_scaling={"rope_type": "longrope"}))
    assert theta is None and "unsupported" in problem
    assert "unsupported" in rope_support(SimpleNamespace(rope_scaling="yarn"))[1]
