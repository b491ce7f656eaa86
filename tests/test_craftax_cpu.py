"""Craftax on CPU: game rules, observation layout, environment resets, learners, metric, smoke ladder."""

from __future__ import annotations

import torch

from priml_b200.baselines.craftax import (
    ActorCritic,
    ActorCriticGTrXL,
    CraftaxEnv,
    CraftaxGTrXLTrainStep,
    CraftaxPQNTrainStep,
    CraftaxRNNTrainStep,
    CraftaxScore,
    CraftaxTrainStep,
)
from priml_b200.baselines.craftax import experiments
from priml_b200.baselines.craftax.game import constants as C
from priml_b200.baselines.craftax.game import observation, world
from priml_b200.baselines.craftax.game import step as rules
from priml_b200.baselines.craftax.game.constants import Achievement as A
from priml_b200.baselines.craftax.game.constants import Action as Act
from priml_b200.baselines.craftax.game.constants import BlockType as B
from priml_b200.baselines.craftax.metric import crafter_score_pct
from priml_b200.parallel.strategies import NoParallel

CPU = torch.device("cpu")


def _world(n: int = 2, seed: int = 0):  # noqa: ANN202
    s = world.generate(n, generator=torch.Generator().manual_seed(seed), device=CPU)
    s.passive.mask[:] = False  # no creatures in the way of scripted tests
    return s


def _act(s, a: Act):  # noqa: ANN001, ANN202
    return rules.step(s, torch.full((s.num_envs,), int(a)), generator=torch.Generator().manual_seed(1))


def _face(s, block: B) -> None:  # noqa: ANN001
    """Put ``block`` right of the player and face it."""
    r, c = s.position[0].tolist()
    s.map[:, r, c + 1] = int(block)
    s.direction[:] = int(Act.RIGHT)


def test_constants_and_observation_layout() -> None:
    assert C.REWARD_CEILING == 226.0 and len(Act) == 43 and C.NUM_ACHIEVEMENTS == 67
    s = _world()
    o = observation.render(s)
    assert o.shape == (2, 8268) == (2, observation.observation_size())
    tiles = o[:, : 9 * 11 * observation.CHANNELS_PER_TILE].view(2, 9, 11, -1)
    assert torch.all(tiles[:, 4, 5, int(B.GRASS)] == 1)  # the player stands on cleared grass at the centre
    assert torch.all(tiles[..., -1] == 1)  # the overworld is lit
    assert torch.allclose(tiles[..., : len(B)].sum(-1), torch.ones(2, 9, 11))


def test_world_generation_is_seeded_and_has_resources() -> None:
    a, b = _world(8, 3), _world(8, 3)
    assert torch.equal(a.map, b.map)
    counts = torch.bincount(a.map.flatten(), minlength=len(B))
    for block in (B.GRASS, B.WATER, B.STONE, B.TREE, B.COAL, B.SAND):
        assert counts[int(block)] > 0, block


def test_tools_gate_mining_and_crafting_needs_a_table() -> None:
    s = _world(1)
    _face(s, B.TREE)
    for _ in range(3):
        s, r = _act(s, Act.DO)
    assert int(s.wood) == 3 and bool(s.achievements[0, A.COLLECT_WOOD])
    _face(s, B.STONE)
    s, _ = _act(s, Act.DO)
    assert int(s.stone) == 0  # no pickaxe yet
    s, _ = _act(s, Act.MAKE_WOOD_PICKAXE)
    assert int(s.pickaxe) == 0  # no table nearby
    _face(s, B.GRASS)
    s, reward = _act(s, Act.PLACE_TABLE)
    assert bool(s.achievements[0, A.PLACE_TABLE]) and float(reward) >= 1.0
    s, _ = _act(s, Act.MAKE_WOOD_PICKAXE)
    assert int(s.pickaxe) == 1 and bool(s.achievements[0, A.MAKE_WOOD_PICKAXE])
    _face(s, B.STONE)
    s, _ = _act(s, Act.DO)
    assert int(s.stone) == 1 and bool(s.achievements[0, A.COLLECT_STONE])
    r, c = s.position[0].tolist()
    assert int(s.map[0, r, c + 1]) == int(B.PATH)
    _face(s, B.IRON)
    s, _ = _act(s, Act.DO)
    assert int(s.iron) == 0  # iron needs a stone pickaxe


def test_water_drink_sleep_and_survival_meters() -> None:
    s = _world(1)
    s.drink[:] = 3
    _face(s, B.WATER)
    s, _ = _act(s, Act.DO)
    assert int(s.drink) == 4 and bool(s.achievements[0, A.COLLECT_DRINK])
    s.energy[:] = 5
    s, _ = _act(s, Act.SLEEP)
    assert bool(s.sleeping)
    for _ in range(120):
        if not bool(s.sleeping):
            break
        s.melee.mask[:] = False
        s, _ = _act(s, Act.NOOP)
    assert not bool(s.sleeping) and bool(s.achievements[0, A.WAKE_UP])
    t = _world(1)
    t.melee.mask[:] = False
    for _ in range(30):
        t.melee.mask[:] = False
        t, _ = _act(t, Act.NOOP)
    assert int(t.food) == C.MAX_METER - 1  # hunger crossed 25 once
    assert int(t.drink) == C.MAX_METER - 1  # thirst crossed 20 once


def test_cow_is_eaten_and_zombie_attacks() -> None:
    s = _world(1)
    r, c = s.position[0].tolist()
    s.passive.mask[0, 0] = True
    s.passive.position[0, 0] = torch.tensor([r, c + 1])
    s.passive.health[0, 0] = 1.0
    s.direction[:] = int(Act.RIGHT)
    s.food[:] = 2
    s, _ = _act(s, Act.DO)
    assert bool(s.achievements[0, A.EAT_COW]) and int(s.food) == 8 and not bool(s.passive.mask[0, 0])
    s.melee.mask[0, 0] = True
    s.melee.position[0, 0] = torch.tensor([r + 1, c])
    s.melee.health[0, 0] = 5.0
    s.melee.cooldown[0, 0] = 0
    h = float(s.health)
    s, reward = _act(s, Act.NOOP)
    assert float(s.health) < h and float(reward) < 0


def test_env_auto_resets_and_state_round_trips() -> None:
    env = CraftaxEnv.Config(num_envs=4, device="cpu", seed=0, optimistic_reset_ratio=2).make()
    obs = env.reset()
    assert obs.shape == (4, 8268)
    env.state.health[1] = 0.0
    t = env.step(torch.zeros(4, dtype=torch.long))
    assert bool(t.done[1]) and not bool(t.done[0])
    assert int(env.state.timestep[1]) == 0 and float(env.state.health[1]) == C.MAX_METER  # a fresh world
    saved = env.state_dict()
    a = env.step(torch.full((4,), int(Act.DO))).observation
    env.load_state_dict(saved)
    b = env.step(torch.full((4,), int(Act.DO))).observation
    assert torch.equal(a, b)


def _step_cfg(cls, **kw):  # noqa: ANN001, ANN202
    c = cls.Config()
    c.env = CraftaxEnv.Config(num_envs=4, device="cpu", seed=0)
    c.parallelism = NoParallel.Config(device="cpu")
    c.dtype_autocast = None
    c.model.hidden_size = 32
    c.rollout_steps = 8
    c.num_minibatches = 2
    c.num_epochs = 2
    c.total_train_steps = 10
    for k, v in kw.items():
        setattr(c, k, v)
    return c.make()


def test_ppo_recurrent_ppo_and_pqn_update() -> None:
    for cls in (CraftaxTrainStep, CraftaxRNNTrainStep, CraftaxGTrXLTrainStep, CraftaxPQNTrainStep):
        kw = {"rollout_steps": 8}
        step = _step_cfg(cls, **kw)
        if cls is CraftaxGTrXLTrainStep:
            step = _step_cfg(cls, model=ActorCriticGTrXL.Config(embed_dim=32, num_heads=4, hidden_size=32,
                                                                 memory_length=8))  # fmt: skip
        before = [p.detach().clone() for p in step.model.parameters()]
        out = step.train_step()
        assert torch.isfinite(out["loss"]).all() and out["stepped"], cls.__name__
        assert any(not torch.equal(a, b) for a, b in zip(before, step.model.parameters(), strict=True))
        step._lr()
        assert step.global_step == 1 and abs(step.optimizer.param_groups[0]["lr"] - 3e-4 * 0.9) < 1e-12  # annealed
        state = step.state_dict()
        again = _step_cfg(cls, model=step.config.model.copy_tree()) if cls is CraftaxGTrXLTrainStep else _step_cfg(cls)
        again.load_state_dict(state)
        assert again.global_step == 1


def test_crafter_score_and_metric_plays_a_policy() -> None:
    assert crafter_score_pct([0.0] * 5) == 0.0
    assert abs(crafter_score_pct([100.0] * 3) - 100.0) < 1e-9
    metric = CraftaxScore(CraftaxScore.Config(num_envs=3, steps=60, device="cpu"))
    policy = ActorCritic.Config(hidden_size=16).make()
    metric.update(None, policy=policy)
    res = metric.compute()
    assert "episodes" in res


def test_experiment_chain_and_smoke_loop(tmp_path) -> None:  # noqa: ANN001
    for exp in (experiments.exp000, experiments.exp001, experiments.exp002, experiments.exp003, experiments.exp011,
                experiments.exp013):
        cfg = exp().copy_tree().finalize()
        assert cfg.step.total_train_steps > 0
    assert experiments.exp000().step.total_train_steps == 244
    cfg = experiments.exp_smoke()
    cfg.step.env.device = "cpu"
    cfg.step.parallelism = NoParallel.Config(device="cpu")
    cfg.step.dtype_autocast = None
    cfg.step.model.hidden_size = 16
    cfg.metrics["craftax"].device = "cpu"
    cfg.base_dir = str(tmp_path)
    loop = cfg.make()
    loop.run()
    assert loop.global_step == 3
    assert "eval/craftax_episodes" in loop.last_eval or "eval/total_loss" in loop.last_eval


def test_ladders_need_kills_and_the_dungeon_is_dark() -> None:
    s = _world(2)
    s.position = s.ladder_down[:, 0].clone()
    s, _ = _act(s, Act.DESCEND)
    assert s.level.tolist() == [0, 0]  # the floor is not cleared yet
    s.kills[:, 0] = C.MONSTERS_KILLED_TO_CLEAR_LEVEL
    s, reward = _act(s, Act.DESCEND)
    assert s.level.tolist() == [1, 1] and bool(s.achievements[:, A.ENTER_DUNGEON].all()) and s.xp.tolist() == [1, 1]
    assert torch.equal(s.position, s.ladder_up[:, 1]) and bool((reward >= 3).all())
    tiles = observation.render(s)[:, : 9 * 11 * observation.CHANNELS_PER_TILE].view(2, 9, 11, -1)
    lit = tiles[..., -1]
    assert int(lit.sum()) == 2 * 7 * 7  # only the 7 x 7 around the player
    s, _ = _act(s, Act.ASCEND)
    assert s.level.tolist() == [0, 0] and torch.equal(s.position, s.ladder_down[:, 0])
    s, _ = _act(s, Act.DESCEND)
    assert s.xp.tolist() == [1, 1]  # experience only for the first visit


def test_chest_bow_arrow_potion_and_level_up() -> None:
    s = _world(1)
    s.level[:] = 1
    _face(s, B.CHEST)
    s, _ = _act(s, Act.DO)
    assert bool(s.achievements[0, A.OPEN_CHEST]) and bool(s.achievements[0, A.FIND_BOW]) and int(s.bow) == 1
    assert int(s.arrows) >= 1
    r, c = s.position[0].tolist()
    s.map[0, r, c + 1 : c + 4] = int(B.PATH)
    s.melee.mask[0, 0] = True
    s.melee.position[0, 0] = torch.tensor([r, c + 2])
    s.melee.health[0, 0] = 1.0
    s.melee.cooldown[0, 0] = 99
    s.arrows[:] = 3
    s, _ = _act(s, Act.SHOOT_ARROW)
    for _ in range(3):
        if not bool(s.melee.mask[0, 0]):
            break
        s.melee.position[0, 0] = torch.tensor([r, c + 2])  # hold the target still
        s, _ = _act(s, Act.NOOP)
    assert bool(s.achievements[0, A.FIRE_BOW]) and not bool(s.melee.mask[0, 0])
    assert bool(s.achievements[0, A.DEFEAT_ORC_SOLIDER]) and int(s.kills[0, 1]) == 1
    s.potions[0, 2] = 1
    s, _ = _act(s, Act.DRINK_POTION_BLUE)
    assert bool(s.achievements[0, A.DRINK_POTION]) and int(s.potions[0, 2]) == 0
    s.xp[:] = 1
    s, _ = _act(s, Act.LEVEL_UP_STRENGTH)
    assert int(s.strength) == 2 and int(s.xp) == 0


def test_nine_floors_entry_achievements_and_gems() -> None:
    s = _world(1)
    assert s.floor_map.shape[1] == C.LEVELS == 9
    assert int((s.floor_items[0, C.LEVELS - 1] == int(C.ItemType.LADDER_DOWN)).sum()) == 0  # the graveyard is last
    for level in range(C.LEVELS - 1):
        s.position = s.ladder_down[:, level].clone()
        s.kills[:, level] = C.MONSTERS_KILLED_TO_CLEAR_LEVEL
        s, _ = _act(s, Act.DESCEND)
        assert s.level.tolist() == [level + 1] and bool(s.achievements[0, C.LEVEL_ACHIEVEMENT[level + 1]])
    assert int(s.xp) == C.LEVELS - 1
    lit = observation.render(s)[:, : 9 * 11 * observation.CHANNELS_PER_TILE].view(1, 9, 11, -1)[..., -1]
    assert int(lit.sum()) == 9 * 11  # the graveyard is lit throughout
    _face(s, B.SAPPHIRE)
    s.pickaxe[:] = 3
    s, _ = _act(s, Act.DO)
    assert int(s.sapphire) == 0  # a diamond pickaxe is needed
    s.pickaxe[:] = 4
    s, _ = _act(s, Act.DO)
    assert int(s.sapphire) == 1 and bool(s.achievements[0, A.COLLECT_SAPPHIRE])
    # the troll mines' deep things throw harder than the overworld's skeletons
    s.level[:] = 5
    assert float(rules._species_damage(s, 2, 1).sum()) > sum(C.SPECIES_DAMAGE[0][1])


def test_books_spells_enchanting_and_the_necromancer() -> None:
    s = _world(1)
    s.level[:] = 3
    _face(s, B.CHEST)
    s, _ = _act(s, Act.DO)
    assert int(s.books) == 1  # the sewers' first chest holds a spellbook
    s, _ = _act(s, Act.READ_BOOK)
    assert bool(s.spells[0, 0]) and bool(s.achievements[0, A.LEARN_FIREBALL]) and int(s.books) == 0
    r, c = s.position[0].tolist()
    s.map[0, r, c + 1 : c + 4] = int(B.PATH)
    s.melee.mask[0, 0] = True
    s.melee.position[0, 0] = torch.tensor([r, c + 2])
    s.melee.health[0, 0] = 5.0
    s.melee.cooldown[0, 0] = 99
    mana = int(s.mana)
    s, _ = _act(s, Act.CAST_FIREBALL)
    assert bool(s.achievements[0, A.CAST_FIREBALL]) and int(s.mana) == mana - 2
    for _ in range(3):
        if not bool(s.melee.mask[0, 0]):
            break
        s.melee.position[0, 0] = torch.tensor([r, c + 2])
        s, _ = _act(s, Act.NOOP)
    assert not bool(s.melee.mask[0, 0])  # 6 spell damage beats 5 health in one hit
    # enchanting at a fire table spends a ruby and 9 mana
    _face(s, B.ENCHANTMENT_TABLE_FIRE)
    s.sword[:], s.ruby[:], s.mana[:] = 1, 1, 9
    before = rules._player_damage(s)
    s, _ = _act(s, Act.ENCHANT_SWORD)
    assert int(s.sword_enchant) == 1 and int(s.ruby) == 0 and int(s.mana) <= 1 and bool(s.achievements[0, A.ENCHANT_SWORD])
    after = rules._player_damage(s)
    assert float(after[0, 1]) > 0 and float(before[0, 1]) == 0 and float(after[0, 0]) == float(before[0, 0])
    s.armour[0] = torch.tensor([1, 0, 0, 0])
    s.sapphire[:], s.mana[:] = 1, 9
    _face(s, B.ENCHANTMENT_TABLE_ICE)
    s, _ = _act(s, Act.ENCHANT_ARMOUR)
    assert s.armour_enchant[0].tolist() == [2, 0, 0, 0] and bool(s.achievements[0, A.ENCHANT_ARMOUR])
    # the necromancer: struck only while nothing it summoned lives and it is not summoning
    s = _world(1)
    last = C.LEVELS - 1
    s.map, s.item_map, s.level[:] = s.floor_map[:, last].clone(), s.floor_items[:, last].clone(), last
    assert int((s.map == int(B.NECROMANCER)).sum()) == 1
    s.melee.mask[:] = False
    s.ranged.mask[:] = False
    _face(s, B.NECROMANCER)
    s, _ = _act(s, Act.DO)
    assert int(s.boss_progress) == 1 and bool(s.achievements[0, A.DAMAGE_NECROMANCER]) and int(s.boss_wait) > 0
    s, _ = _act(s, Act.DO)
    assert int(s.boss_progress) == 1  # summoning: shielded
    s.boss_progress[:] = last
    s, reward = _act(s, Act.NOOP)
    assert bool(s.achievements[0, A.DEFEAT_NECROMANCER]) and float(reward) >= 8 and bool(rules.is_done(s))
    obs = observation.render(s)
    assert obs.shape[-1] == observation.observation_size() and torch.isfinite(obs).all()


def test_bench_prints_env_steps_per_second(capsys, monkeypatch) -> None:  # noqa: ANN001
    import json
    import sys

    from priml_b200.baselines.craftax import bench

    monkeypatch.setattr(sys, "argv", ["bench", "--device", "cpu", "--envs", "8", "--rollout", "2", "--steps", "1"])
    bench.main()
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["unit"] == "steps/s" and line["value"] > 0


def test_pixel_renderer_layers_and_shading(tmp_path) -> None:  # noqa: ANN001
    """Frames are the 9 x 11 view in tiles of P pixels; sprites from a folder replace the stand-ins;
    sleep halves the brightness, night fades toward blue, unseen tiles are black."""
    from torchvision.io import write_png

    from priml_b200.baselines.craftax.game import constants as C
    from priml_b200.baselines.craftax.game import world
    from priml_b200.baselines.craftax.game.pixels import PixelRenderer

    s = world.generate(3, generator=torch.Generator().manual_seed(0), device=torch.device("cpu"))
    red = torch.zeros(3, 8, 8, dtype=torch.uint8)
    red[0] = 255
    write_png(red, str(tmp_path / "grass.png"))
    r = PixelRenderer(block_pixels=8, sprite_dir=tmp_path)
    assert r.found == ["grass.png"]
    frame = r.render(s)
    assert frame.shape == (3, 9 * 8, 11 * 8, 3) and frame.dtype == torch.uint8
    assert torch.equal(frame, r.render(s))  # deterministic

    from priml_b200.baselines.craftax.game.observation import local_view

    blocks, _ = local_view(s)
    grass = (blocks[0] == int(C.BlockType.GRASS)).nonzero()
    assert len(grass) > 0
    for row, col in grass.tolist()[:5]:
        if (row, col) == (4, 5):
            continue  # the player stands here
        tile = frame[0, row * 8 : row * 8 + 8, col * 8 : col * 8 + 8]
        # daylight may dim the frame a little, but grass stays red-dominated
        assert (tile[..., 0].float() > tile[..., 1].float() + 50).all()

    s.sleeping[1] = True
    s.light[2] = 0.0
    dimmed = r.render(s)
    away = torch.ones(9 * 8, 11 * 8, dtype=torch.bool)
    away[4 * 8 : 5 * 8, 5 * 8 : 6 * 8] = False  # the player's own tile shows the sleeping sprite
    assert (dimmed[1].float() <= frame[1].float() * 0.5 + 1)[away].all()
    night = torch.tensor([0, 16, 64], dtype=torch.float32)
    assert ((dimmed[2].float() - night).abs() <= 1).all()  # fully dark surface is the night colour

    # a player in a dark cave sees only the tiles near it
    s.level[0] = 1
    s.map[0] = s.floor_map[0, 1]
    s.item_map[0] = torch.zeros_like(s.item_map[0])
    cave = r.render(s)
    assert cave[0, :8, :8].max() == 0  # the corner tile is 4+ tiles away: unseen
    PixelRenderer.write_png(cave[0], tmp_path / "frame.png")
    assert (tmp_path / "frame.png").stat().st_size > 0


def test_elemental_damage_and_resistance() -> None:
    """Fire-realm creatures shrug off fire and most physical damage; enchanted armour blocks its element."""
    s = _world(1)
    s.level[:] = 6  # the fire realm: pigmen and fire elementals
    hit = rules._species_damage(s, 1, 0)[0].tolist()
    assert hit[1] > 0 and hit[2] == 0  # a pigman's blow carries fire
    fire = rules._in_element(torch.tensor([6.0]), torch.tensor([1]))
    ice = rules._in_element(torch.tensor([6.0]), torch.tensor([2]))
    defense = rules._species_defense(s, 1)
    assert float(((1 - defense) * fire).sum()) == 0.0  # immune to a fireball
    assert float(((1 - defense) * ice).sum()) == 6.0  # an iceball lands in full
    # a fire-enchanted piece blocks a fifth of a fire blow's fire share, nothing of its physical share
    s.armour[0] = torch.tensor([1, 0, 0, 0])
    plain = float(rules._damage_to_player(s, torch.tensor([[0.0, 5.0, 0.0]])))
    s.armour_enchant[0] = torch.tensor([1, 0, 0, 0])
    warded = float(rules._damage_to_player(s, torch.tensor([[0.0, 5.0, 0.0]])))
    assert abs(plain - 5.0) < 1e-6 and abs(warded - 4.0) < 1e-6
    assert abs(float(rules._damage_to_player(s, torch.tensor([[10.0, 0.0, 0.0]]))) - 9.0) < 1e-6
