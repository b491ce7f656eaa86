"""Sudoku baseline on CPU: model lattice, recurrence, prefix, ACT pool, data, metric, train step."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from priml_b200.baselines.sudoku import (
    ActPool,
    DeepRecurrence,
    FactoredPositions,
    GridAccuracy,
    GridEmbedding,
    PredictionFeedback,
    PrefixStack,
    RegisterTokens,
    SparsePuzzleEmbedding,
    SudokuNet,
    SudokuTrainStep,
    augment_sudoku,
)
from priml_b200.baselines.sudoku import experiments, prepare_data
from priml_b200.models.norm import RMSNorm
from priml_b200.models.swiglu import SwiGLU
from priml_b200.models.transformer import TransformerBlock
from priml_b200.models.vision import MLPMixerBlock
from priml_b200.optimizers import SignSGD
from priml_b200.parallel.strategies import NoParallel


def _solution(rng: np.random.Generator) -> np.ndarray:
    """A valid solved grid (0-based pattern shifted to digits 1..9), then a random transform."""
    r, c = np.meshgrid(np.arange(9), np.arange(9), indexing="ij")
    base = (3 * (r % 3) + r // 3 + c) % 9 + 1
    return prepare_data.transform(base, base, rng)[1]


def _valid(grid: np.ndarray) -> bool:
    want = set(range(1, 10))
    rows = all(set(grid[i]) == want for i in range(9))
    cols = all(set(grid[:, j]) == want for j in range(9))
    boxes = all(set(grid[3 * a : 3 * a + 3, 3 * b : 3 * b + 3].reshape(-1)) == want for a in range(3) for b in range(3))
    return rows and cols and boxes


def _puzzle(sol: np.ndarray, rng: np.random.Generator, blanks: int = 40) -> np.ndarray:
    p = sol.copy()
    p.reshape(-1)[rng.choice(81, blanks, replace=False)] = 0
    return p


def _config(*, recurrent: bool = False, mixer: bool = False, prefix: bool = False) -> SudokuNet.Config:
    c = SudokuNet.Config(hidden_size=16, num_layers=1)
    c.embedding = GridEmbedding.Config()
    c.block = TransformerBlock.Config(prenorm=False, ffn=SwiGLU.Config(round_to=16))
    if mixer:
        c.block = MLPMixerBlock.Config(seq_len=81 + (3 if prefix else 0), prenorm=False,
                                       token_mixer=SwiGLU.Config(norm=RMSNorm.Config(), round_to=16),
                                       channel_mixer=SwiGLU.Config(norm=RMSNorm.Config(), round_to=16))  # fmt: skip
    if recurrent:
        c.recurrence = DeepRecurrence.Config(slow_cycles=2, fast_cycles=2)
    if prefix:
        c.prefix = PrefixStack.Config(parts=[SparsePuzzleEmbedding.Config(num_puzzles=5, num_tokens=2, batch_size=2),
                                             RegisterTokens.Config(num_tokens=1)])  # fmt: skip
    return c


@pytest.mark.parametrize("mixer", [False, True])
@pytest.mark.parametrize("recurrent", [False, True])
def test_every_corner_of_the_lattice_runs(mixer: bool, recurrent: bool) -> None:
    torch.manual_seed(0)
    out = _config(mixer=mixer, recurrent=recurrent).make()(torch.randint(0, 11, (2, 81)))
    assert out.logits.shape == (2, 81, 11) and out.halt.shape == (2,)
    assert not out.z_slow.requires_grad  # carried latents are detached


def test_recurrence_adds_no_parameters_and_backward_is_flat_in_depth() -> None:
    torch.manual_seed(0)
    plain = sum(p.numel() for p in _config().make().parameters())
    assert plain == sum(p.numel() for p in _config(recurrent=True).make().parameters())

    def graph_nodes(slow: int) -> int:
        torch.manual_seed(0)
        cfg = _config(recurrent=True)
        cfg.recurrence = DeepRecurrence.Config(slow_cycles=slow, fast_cycles=2)
        loss = cfg.make()(torch.randint(0, 11, (2, 81))).logits.sum()
        seen, todo = set(), [loss.grad_fn]
        while todo:
            f = todo.pop()
            if f is None or f in seen:
                continue
            seen.add(f)
            todo.extend(n for n, _ in f.next_functions)
        return len(seen)

    assert graph_nodes(1) == graph_nodes(4)


def test_halt_starts_negative_and_prefix_is_stripped() -> None:
    torch.manual_seed(0)
    cfg = _config(prefix=True)
    m = cfg.make()
    assert m.config.num_prefix_tokens == 3 and m.config.total_seq_len == 84
    m.train()
    out = m(torch.randint(0, 11, (2, 81)), puzzle_identifiers=torch.tensor([1, 4]))
    assert out.logits.shape == (2, 81, 11) and out.z_slow.shape == (2, 84, 16)
    assert torch.allclose(out.halt, torch.full((2,), -5.0))
    out.logits.float().sum().backward()
    table = m.prefix.parts[0]
    assert table.local_weights.grad is not None and table.local_weights.grad.shape == (2, 16)
    assert table.local_ids.tolist() == [1, 4]


def test_sparse_embedding_is_inert_at_zero_init_and_sign_sgd_updates_only_its_rows() -> None:
    cfg = SparsePuzzleEmbedding.Config(num_puzzles=6, num_tokens=2, hidden_size=4, batch_size=3)
    emb = cfg.make()
    emb.train()
    out = emb(3, puzzle_identifiers=torch.tensor([0, 2, 2]))
    assert out.shape == (3, 2, 4) and float(out.detach().abs().sum()) == 0.0
    out.sum().backward()
    opt = SignSGD([{"params": [emb.weights, emb.local_weights, emb.local_ids], "sparse_embedding": True}], lr=0.5)
    opt.step()
    w = emb.weights
    assert torch.all(w[[0, 2]] == -0.5) and torch.all(w[[1, 3, 4, 5]] == 0)


def test_feedback_channel_is_one_shot() -> None:
    ch = PredictionFeedback.Config(vocab_size=11, hidden_size=8, init_std=1.0).make()
    e = torch.zeros(1, 81, 8)
    assert ch(None, e).numel() == 0
    ch.set_feedback(torch.ones(1, 81, dtype=torch.long))
    assert ch(None, e).shape == (1, 81, 8)
    assert ch(None, e).numel() == 0


def test_factored_positions_share_rows_columns_and_boxes() -> None:
    pos = FactoredPositions.Config(hidden_size=8).make()
    assert pos.box_index.view(9, 9)[0].tolist() == [0, 0, 0, 1, 1, 1, 2, 2, 2]
    assert pos.box_index.view(9, 9)[4, 4] == 4
    with pytest.raises(ValueError, match="does not tile"):
        FactoredPositions.Config(grid_shape=(9, 9), box_shape=(2, 3), hidden_size=8).make()


def _pool(n: int = 4, max_steps: int = 3, prob: float = 0.0) -> ActPool:
    return ActPool.Config(batch_size=n, max_steps=max_steps, grid_len=81, seq_len=81, hidden_size=8,
                          halt_exploration_prob=prob).make()  # fmt: skip


def test_act_pool_refills_only_halted_slots_and_halts_at_the_cap() -> None:
    pool = _pool()
    a = torch.full((4, 81), 2)
    inputs, labels, active = pool.refill(a, labels=a, valid_count=3, ignore_label_id=-100)
    assert torch.equal(inputs, a) and bool(active.all())
    assert torch.all(labels[3] == -100)  # padding rows are never scored
    z = torch.ones(4, 81, 8)
    pool.advance(z, z_fast=z, logits=torch.zeros(4, 81, 11), halt=torch.tensor([1.0, -1.0, -1.0, -1.0]), media=inputs)
    assert pool.halted.tolist() == [True, False, False, False]
    b = torch.full((4, 81), 3)
    inputs, _, _ = pool.refill(b, labels=b, valid_count=4, ignore_label_id=-100)
    assert inputs[0, 0] == 3 and inputs[1, 0] == 2  # only the halted slot was re-seated
    assert pool.z_slow[0].abs().sum() == 0 and pool.z_slow[1].abs().sum() > 0
    for _ in range(3):
        pool.advance(z, z_fast=z, logits=torch.zeros(4, 81, 11), halt=torch.full((4,), -1.0), media=inputs)
    assert bool(pool.halted[1:].all())  # step cap reached


def test_givens_survive_the_feedback_loop_and_only_the_rng_is_checkpointed() -> None:
    pool = _pool(prob=0.5)
    media = torch.tensor([[1, 5] + [1] * 79] * 4)
    decoded = torch.full((4, 81), 7)
    fed = pool.clamp_givens(decoded, media=media)
    assert fed[0, 1] == 5 and fed[0, 0] == 7
    assert set(pool.state_dict()) == {"halt_rng"}
    s = pool.state_dict()
    first = torch.rand(3, generator=pool._generator)
    pool.load_state_dict(s)
    assert torch.equal(first, torch.rand(3, generator=pool._generator))


def test_augmentation_and_transforms_preserve_validity() -> None:
    rng = np.random.default_rng(0)
    sols = np.stack([_solution(rng) for _ in range(6)])
    assert all(_valid(s) for s in sols)
    tok = torch.from_numpy(sols.reshape(6, 81) + 1)
    g = torch.Generator().manual_seed(0)
    x, y = augment_sudoku(tok, tok, generator=g)
    assert torch.equal(x, y)
    assert all(_valid(s) for s in (y - 1).view(6, 9, 9).numpy())
    assert not torch.equal(y, tok)


def _write_dataset(root, n_train: int = 6, n_test: int = 4, copies: int = 3) -> None:  # noqa: ANN001
    rng = np.random.default_rng(1)
    for split, n, k in (("train", n_train, copies), ("test", n_test, 0)):
        sols = [_solution(rng) for _ in range(n)]
        prepare_data.write_split(root / split, [_puzzle(s, rng) for s in sols], sols, copies_per_puzzle=k, rng=rng)


def test_prepared_split_loads_and_pads_the_last_batch(tmp_path) -> None:  # noqa: ANN001
    _write_dataset(tmp_path)
    from priml_b200.baselines.sudoku.data import SudokuData

    data = SudokuData.Config(working_dir=str(tmp_path), batch_size=5, device="cpu", seed=0).make()
    batches = list(data.train_dataloader())
    assert len(batches) == 5 and batches[-1]["valid_count"] == 4  # 24 rows
    assert all(b["media"].shape == (5, 81) for b in batches)
    for b in batches:
        sol = (b["label"][: b["valid_count"]] - 1).view(-1, 9, 9).numpy()
        assert all(_valid(s) for s in sol)
        given = b["media"] >= 2
        assert torch.equal(b["media"][given], b["label"][given])
    ev = list(data.eval_dataloader())
    assert sum(b["valid_count"] for b in ev) == 4


def test_grid_accuracy_counts_whole_grids_and_cells() -> None:
    m = GridAccuracy()
    labels = torch.tensor([[2, 3, 4], [2, 3, 4], [5, 5, 5]])
    packed = torch.tensor([[-1.0, 2, 3, 4], [0.5, 2, 3, 9], [0.0, 0, 0, 0]])
    m.update(packed, label=labels, valid_count=2)
    assert m.compute() == {"exact": 0.5, "cell": 5 / 6}


def _step(*, act: bool = False, feedback: bool = False) -> SudokuTrainStep:
    c = SudokuTrainStep.Config()
    c.parallelism = NoParallel.Config(device="cpu")
    c.dtype_autocast = None
    c.model = _config(recurrent=act)
    if feedback:
        c.model.embedding.channels = [PredictionFeedback.Config()]
    c.total_train_steps = 50
    if act:
        c.act = ActPool.Config(batch_size=8, max_steps=2)
    torch.manual_seed(0)
    return c.make()


def _batch(seed: int = 0) -> dict[str, object]:
    rng = np.random.default_rng(seed)
    sols = [_solution(rng) for _ in range(8)]
    media = torch.from_numpy(np.stack([_puzzle(s, rng) for s in sols]).reshape(8, 81) + 1)
    return {"media": media, "label": torch.from_numpy(np.stack(sols).reshape(8, 81) + 1), "valid_count": 8}


def test_train_step_learns_and_reports_act_metrics() -> None:
    step = _step()
    batch = _batch()
    losses = [float(step.train_step(**batch)["loss"]) for _ in range(15)]
    assert losses[-1] < losses[0]
    assert "halt_loss" not in step.train_step(**batch)["metrics"]
    rec = _step(act=True).train_step(**batch)["metrics"]
    assert {"halt_loss", "halted_frac", "act_steps", "lm_loss", "lr"} <= set(rec)


def test_state_round_trips_including_ema() -> None:
    step = _step()
    step.train_step(**_batch())
    state = step.state_dict()
    restored = _step()
    restored.load_state_dict(state)
    assert restored.global_step == step.global_step == 1
    for (n, a), (_, b) in zip(step.model.named_parameters(), restored.model.named_parameters(), strict=True):
        assert torch.equal(a, b), n
    for n, v in step.ema_shadow.items():
        assert torch.equal(restored.ema_shadow[n], v)


def test_eval_rollout_packs_halt_and_grid_and_consumes_feedback() -> None:
    step = _step(act=True, feedback=True)
    step.train_step(**_batch())
    out = step.eval_loss(**_batch(1))
    assert out["model"].shape == (8, 82)
    ch = step.model.embedding.channels[0]
    assert ch._ids is None  # consumed by the last rollout step, never left stashed
    m = GridAccuracy()
    m.update(out["model"], **_batch(1))
    assert 0.0 <= m.compute()["cell"] <= 1.0


def test_puzzle_optimizer_trains_the_sparse_table() -> None:
    c = SudokuTrainStep.Config()
    c.parallelism = NoParallel.Config(device="cpu")
    c.dtype_autocast = None
    c.model = _config(prefix=True)
    c.total_train_steps = 10
    c.puzzle_optimizer = SignSGD.Config(lr=0.01)
    torch.manual_seed(0)
    step = c.make()
    b = _batch()
    batch = {"media": b["media"][:2], "label": b["label"][:2], "valid_count": 2,
             "puzzle_identifiers": torch.tensor([1, 3])}  # fmt: skip
    step.train_step(**batch)
    table = step.model.prefix.parts[0].weights
    assert table[[1, 3]].abs().sum() > 0 and table[[0, 2, 4]].abs().sum() == 0


def test_horizon_must_be_positive() -> None:
    c = SudokuTrainStep.Config()
    c.total_train_steps = 0
    with pytest.raises(ValueError, match="total_train_steps must be positive"):
        c.make()


def test_experiment_ladder_and_smoke_run(tmp_path) -> None:  # noqa: ANN001
    for exp in (experiments.exp000, experiments.exp001, experiments.exp002, experiments.exp003):
        cfg = exp().copy_tree().finalize()
        assert cfg.step.model.hidden_size == 512
    assert experiments.exp002().step.act is not None and experiments.exp000().step.act is None
    _write_dataset(tmp_path, n_train=4, n_test=4, copies=2)
    cfg = experiments.exp_smoke()
    cfg.dataset.working_dir = str(tmp_path)
    cfg.dataset.device = "cpu"
    cfg.step.parallelism = NoParallel.Config(device="cpu")
    cfg.step.dtype_autocast = None
    cfg.base_dir = str(tmp_path)
    loop = cfg.make()
    res = loop.run()
    assert loop.global_step == 4
    assert "eval/accuracy_exact" in res or "eval/accuracy_exact" in loop.last_eval
