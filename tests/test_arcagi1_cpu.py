"""ARC-AGI-1 baseline on CPU: task-weighted sampling, pass@K, grid encoding, the smoke ladder."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from priml_b200.baselines.arcagi1 import ArcData, PassK
from priml_b200.baselines.arcagi1 import experiments, prepare_data
from priml_b200.parallel.strategies import NoParallel


def _task(rng: np.random.Generator, n_train: int = 3, n_test: int = 1) -> dict[str, object]:
    """A colour-swap rule: output = input with colours 1 and 2 exchanged."""
    def pair() -> dict[str, list[list[int]]]:
        h, w = (int(v) for v in rng.integers(2, 6, size=2))
        x = rng.integers(0, 4, size=(h, w))
        y = np.where(x == 1, 2, np.where(x == 2, 1, x))
        return {"input": x.tolist(), "output": y.tolist()}
    return {"train": [pair() for _ in range(n_train)], "test": [pair() for _ in range(n_test)]}


@pytest.fixture
def arc_dir(tmp_path):  # noqa: ANN001, ANN201
    rng = np.random.default_rng(0)
    prepare_data.prepare(tmp_path, training=[_task(rng) for _ in range(5)], evaluation=[_task(rng) for _ in range(3)],
                         views=3, seed=0)  # fmt: skip
    return tmp_path


def test_grid_encoding_marks_the_grid_edge() -> None:
    tok = prepare_data.encode_grid(np.array([[0, 9], [3, 4], [5, 6]])).reshape(30, 30)
    assert tok[0, :2].tolist() == [2, 11] and tok[0, 2] == 1 and tok[3, :3].tolist() == [1, 1, 1]
    assert tok[4:].sum() == 0 and tok[:, 3:].sum() == 0
    g = np.arange(6).reshape(2, 3) % 10
    colors = np.arange(10)
    assert np.array_equal(prepare_data.view_transform(g, 1, colors), g[:, ::-1])
    assert prepare_data.view_transform(g, 2, colors).shape == (3, 2)


def test_layout_and_task_weighted_batches(arc_dir) -> None:  # noqa: ANN001
    assert experiments.num_puzzle_identifiers(arc_dir) == 8 * 3
    data = ArcData.Config(working_dir=str(arc_dir), device="cpu", batch_size=4, seed=0).make()
    batches = list(data.train_dataloader())
    assert batches and all(b["media"].shape == (4, 900) and b["valid_count"] == 4 for b in batches)
    b = batches[0]
    assert b["puzzle_identifiers"].shape == (4,)
    assert int((b["label"] == 0).sum()) == 0 and int((b["label"] == -100).sum()) > 0  # pad is ignored
    # whole views arrive together: consecutive rows share an identifier
    ids = b["puzzle_identifiers"].tolist()
    assert ids[0] == ids[1]
    ev = list(data.eval_dataloader())
    assert sum(e["valid_count"] for e in ev) == 3 * 3  # 3 eval tasks x 3 views x 1 test pair
    # every test identifier was trained on
    train_ids = np.load(arc_dir / "train" / "all__puzzle_identifiers.npy")
    test_ids = np.load(arc_dir / "test" / "all__puzzle_identifiers.npy")
    assert set(test_ids.tolist()) <= set(train_ids.tolist())
    s = data.state_dict()
    assert s["passes"] == 1


def test_pass_at_k_ranks_by_votes_then_confidence() -> None:
    m = PassK(PassK.Config(pass_ks=(1, 2)))
    label = torch.tensor([[2, 3], [2, 3], [2, 3], [4, 4]])
    # puzzle 7: two votes for a wrong grid, one confident vote for the right one
    packed = torch.tensor([[0.0, 2, 2], [0.0, 2, 2], [5.0, 2, 3], [0.0, 4, 4]])
    m.update(packed, label=label, puzzle_identifiers=torch.tensor([7, 7, 7, 9]), valid_count=4)
    assert m.compute() == {"pass@1": 0.5, "pass@2": 1.0}
    m.load_state_dict(m.state_dict())
    assert m.compute()["pass@2"] == 1.0


def test_ladder_configs_and_smoke_run(arc_dir) -> None:  # noqa: ANN001
    for exp in (experiments.exp000, experiments.exp001, experiments.exp002, experiments.exp003):
        cfg = exp()
        cfg.dataset.working_dir = str(arc_dir)
        cfg = cfg.copy_tree().finalize()
        assert cfg.step.model.total_seq_len == 917
        assert cfg.step.model.prefix.parts[0].num_puzzles == 24
    cfg = experiments.exp_smoke()
    cfg.dataset.working_dir = str(arc_dir)
    cfg.dataset.device = "cpu"
    cfg.dataset.num_eval_tasks = 2
    cfg.step.parallelism = NoParallel.Config(device="cpu")
    cfg.step.dtype_autocast = None
    cfg.step.model.block.attn.heads = 2
    cfg.base_dir = str(arc_dir)
    loop = cfg.make()
    loop.run()
    assert loop.global_step == 4
    assert "eval/pass_pass@1" in loop.last_eval


def test_recurrent_arc_step_keeps_each_slot_on_its_own_puzzle(arc_dir) -> None:  # noqa: ANN001
    step_cfg = experiments.exp002().step
    step_cfg.model.prefix.parts[0].num_puzzles = experiments.num_puzzle_identifiers(arc_dir)
    step_cfg.model.hidden_size = 32
    step_cfg.model.num_layers = 1
    step_cfg.model.block.attn.heads = 2
    step_cfg.model.recurrence.slow_cycles = 1
    step_cfg.model.recurrence.fast_cycles = 1
    step_cfg.model.prefix.parts[0].batch_size = 4
    step_cfg.act.batch_size = 4
    step_cfg.parallelism = NoParallel.Config(device="cpu")
    step_cfg.dtype_autocast = None
    step = step_cfg.make()
    data = ArcData.Config(working_dir=str(arc_dir), device="cpu", batch_size=4).make()
    it = iter(data.train_dataloader())
    first, second = next(it), next(it)
    step.train_step(**first)
    kept = ~step.act.halted
    step.train_step(**second)
    # slots that did not halt still carry the first batch's identifiers
    assert torch.equal(step.act.identifiers[kept], first["puzzle_identifiers"][kept])
