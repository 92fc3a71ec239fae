"""The registered op `torch.ops.minicpm5_mk.forward` (minicpm5_mk/torch_op.py), without a GPU: it exists
under the reference op's name (`jax_op("minicpm5_mk::forward", ...)`, plugin/minicpm5_mk/model.py:57-66),
its fake implementation gives tracing the output shapes, and it has no CPU kernel (no CPU fallback)."""
import pytest
import torch

from minicpm5_mk import torch_op
from minicpm5_mk.mk_config import PRESETS


class _FakeEngine:
    def __init__(self, cfg):
        self.cfg = cfg

    def forward(self, ids, bs, seq):  # never reached on CPU
        raise AssertionError("the op must not run on CPU")


def test_op_registered_with_fake_shapes():
    cfg = PRESETS["minicpm5-1b"]
    eid = torch_op.register_engine(_FakeEngine(cfg))
    try:
        assert hasattr(torch.ops.minicpm5_mk, "forward")
        from torch._subclasses.fake_tensor import FakeTensorMode
        with FakeTensorMode():
            ids = torch.empty((4 * 8192,), dtype=torch.int32)
            hid, lg, top1 = torch.ops.minicpm5_mk.forward(ids, eid, 4, 8192)
        assert hid.shape == (4, cfg.hidden) and hid.dtype == torch.bfloat16
        assert lg.shape == (4, cfg.vocab) and lg.dtype == torch.float32
        assert top1.shape == (4,) and top1.dtype == torch.int32
    finally:
        torch_op.unregister_engine(eid)


def test_op_has_no_cpu_kernel():
    eid = torch_op.register_engine(_FakeEngine(PRESETS["tiny-hd96"]))
    try:
        with pytest.raises((NotImplementedError, RuntimeError)):
            torch.ops.minicpm5_mk.forward(torch.zeros((256,), dtype=torch.int32), eid, 1, 256)
    finally:
        torch_op.unregister_engine(eid)


def test_unknown_engine_id():
    from torch._subclasses.fake_tensor import FakeTensorMode
    with pytest.raises(RuntimeError, match="no engine"):
        with FakeTensorMode():
            torch.ops.minicpm5_mk.forward(torch.empty((128,), dtype=torch.int32), 10 ** 9, 1, 128)
