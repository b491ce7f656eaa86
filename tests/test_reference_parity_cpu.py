"""Parity with the reference's own code on the tiny fp32 CPU configuration.

The model: vocab 512, d_model 128, 2 layers, 4 heads x 32, SwiGLU 512, RMSNorm,
RoPE theta 1e4. Data: batch 8 x seq 64 uniform tokens from ``torch.manual_seed(0)``,
targets shifted by one. Optimizer: AdamW lr 3e-4, betas (0.9, 0.95), wd 0.1.

The reference package runs unmodified from ``baseline/_ref`` (see
``priml_b200.testing.reference``). Checked here:

* forward: with the reference's initial weights loaded, the logits are bitwise equal;
* training: 20 AdamW steps give the same losses and weights (fp32 tolerance);
* checkpoints: a reference ``TrainStep.state_dict()`` resumes in this framework
  and the other way round, and both continue on the same curve;
* sharded training: the same 20 steps on two gloo ranks -- the reference's FSDP2
  strategy and this framework's sharded strategy -- follow the single-process curve.
"""

from __future__ import annotations

import io

import pytest
import torch

from priml_b200.testing import run_ranks
from priml_b200.testing.reference import load_reference, reference_available

pytestmark = pytest.mark.skipif(not reference_available(), reason="the reference copy is not present")

STEPS = 20
TOL = {"rtol": 2e-5, "atol": 2e-5}


def _batches(n: int) -> list[torch.Tensor]:
    torch.manual_seed(0)
    return [torch.randint(0, 512, (8, 65)) for _ in range(n)]


def _ref_model_cfg():  # noqa: ANN202
    load_reference()
    from priml.model.attention import SelfAttention
    from priml.model.causal_lm import CausalLM
    from priml.model.norm import RMSNorm
    from priml.model.rope import RoPE
    from priml.model.swiglu import SwiGLU
    from priml.model.transformer import TransformerBlock

    block = TransformerBlock.Config(
        attn=SelfAttention.Config(heads=4, channels_head=32, causal=True, rope=RoPE.Config(32, base=1e4)),
        ffn=SwiGLU.Config(channels_hidden=512),
        norm1=RMSNorm.Config(eps=1e-6),
        norm2=RMSNorm.Config(eps=1e-6),
    )
    return CausalLM.Config(512, channels=128, num_layers=2, block=block, final_norm=RMSNorm.Config(eps=1e-6))


def _ref_step(parallelism=None):  # noqa: ANN001, ANN202
    load_reference()
    from priml.baselines.nanochat.train_step import TokenCrossEntropy
    from priml.optimizers.fused_adamw import FusedAdamW
    from priml.train.parallelism import NoParallel
    from priml.train.train_step import TrainStep

    torch.manual_seed(1234)
    return TrainStep.Config(
        model=_ref_model_cfg(),
        optimizer=FusedAdamW.Config(lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1, compile=False),
        loss=TokenCrossEntropy.Config(),
        parallelism=parallelism if parallelism is not None else NoParallel.Config(device="cpu"),
        compile=None,
    ).make()


def _our_step(parallelism=None):  # noqa: ANN001, ANN202
    from priml_b200.loss import TokenCrossEntropy
    from priml_b200.models.presets import tiny_lm
    from priml_b200.optimizers import FusedAdamW
    from priml_b200.train import TrainStep

    kw = {"parallelism": parallelism} if parallelism is not None else {}
    return TrainStep.Config(
        model=tiny_lm(),
        optimizer=FusedAdamW.Config(lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1),
        loss=TokenCrossEntropy.Config(),
        **kw,
    ).make()


def _through_file(state: dict) -> dict:
    """A checkpoint as a file holds it: serialized, and loaded with ``weights_only=True``."""
    buf = io.BytesIO()
    torch.save(state, buf)
    buf.seek(0)
    return torch.load(buf, weights_only=True)


def _ref_train(step, seqs) -> list[float]:  # noqa: ANN001
    out = []
    for seq in seqs:
        res = step.train_step(tokens=seq[:, :-1], label=seq[:, 1:])
        out.append(float(res["loss"].detach().mean()))
    return out


def _our_train(step, seqs) -> list[float]:  # noqa: ANN001
    out = []
    for seq in seqs:
        res = step.train_step(tokens=seq[:, :-1], targets=seq[:, 1:])
        out.append(float(res["loss"].detach().float().mean()))
    return out


def test_forward_is_bitwise_equal_with_reference_weights() -> None:
    torch.manual_seed(0)
    ref = _ref_model_cfg().make()
    from priml_b200.models.presets import tiny_lm

    ours = tiny_lm().make()
    assert sorted(ref.state_dict()) == sorted(ours.state_dict())
    ours.load_state_dict(ref.state_dict())
    tokens = _batches(1)[0][:, :-1]
    with torch.no_grad():
        assert torch.equal(ref(tokens), ours(tokens))


def test_adamw_curve_and_weights_match_reference() -> None:
    ref, ours = _ref_step(), _our_step()
    ours.model.load_state_dict(ref.model.state_dict())
    seqs = _batches(STEPS)
    ref_losses, our_losses = _ref_train(ref, seqs), _our_train(ours, seqs)
    torch.testing.assert_close(torch.tensor(our_losses), torch.tensor(ref_losses), **TOL)
    assert our_losses[-1] < our_losses[0]
    for (name, a), (_, b) in zip(sorted(ours.model.state_dict().items()), sorted(ref.model.state_dict().items()),
                                 strict=True):  # fmt: skip
        torch.testing.assert_close(a, b, **TOL, msg=name)


@pytest.mark.parametrize("direction", ["reference_to_ours", "ours_to_reference"])
def test_checkpoints_resume_across_frameworks(direction: str) -> None:
    seqs = _batches(15)
    ref, ours = _ref_step(), _our_step()
    ours.model.load_state_dict(ref.model.state_dict())
    if direction == "reference_to_ours":
        _ref_train(ref, seqs[:10])
        resumed = _our_step()
        resumed.load_state_dict(_through_file(ref.state_dict()))
        tail_saved, tail_resumed = _ref_train(ref, seqs[10:]), _our_train(resumed, seqs[10:])
    else:
        _our_train(ours, seqs[:10])
        resumed = _ref_step()
        resumed.load_state_dict(_through_file(ours.state_dict()))
        tail_saved, tail_resumed = _our_train(ours, seqs[10:]), _ref_train(resumed, seqs[10:])
    torch.testing.assert_close(torch.tensor(tail_resumed), torch.tensor(tail_saved), **TOL)


def _ref_rank(rank: int, world: int, steps: int) -> list[float]:
    load_reference()
    import torch.distributed as dist
    from priml.runtime import initialize_global_device_mesh
    from priml.train.parallelism import FullySharded

    initialize_global_device_mesh(backend="gloo", device=torch.device("cpu"), mesh_topology={"dp": world})
    step = _ref_step(FullySharded.Config())
    # every rank builds the same initial weights from the same seed, then FSDP2 shards them
    losses = []
    for seq in _batches(steps):
        res = step.train_step(tokens=seq.chunk(world)[rank][:, :-1], label=seq.chunk(world)[rank][:, 1:])
        t = res["loss"].detach().float().mean()
        dist.all_reduce(t)
        losses.append(float(t) / world)
    return losses


def _our_rank(rank: int, world: int, steps: int) -> list[float]:
    import torch.distributed as dist

    from priml_b200.parallel.fused_fsdp import FusedFullySharded

    torch.manual_seed(1234)
    ref_init = _ref_model_cfg().make().state_dict()  # the reference's initial weights, same seed
    step = _our_step(FusedFullySharded.Config(device="cpu"))
    step.model.load_state_dict(ref_init)
    losses = []
    for seq in _batches(steps):
        res = step.train_step(tokens=seq.chunk(world)[rank][:, :-1], targets=seq.chunk(world)[rank][:, 1:])
        t = res["loss"].detach().float().mean()
        dist.all_reduce(t)
        losses.append(float(t) / world)
    return losses


def test_two_rank_sharded_training_matches_reference() -> None:
    single = _ref_train(_ref_step(), _batches(STEPS))
    ref = run_ranks(_ref_rank, 2, STEPS)
    ours = run_ranks(_our_rank, 2, STEPS)
    for r in range(2):
        torch.testing.assert_close(torch.tensor(ref[r]), torch.tensor(single), rtol=1e-4, atol=1e-4)
        torch.testing.assert_close(torch.tensor(ours[r]), torch.tensor(ref[r]), rtol=1e-4, atol=1e-4)
