"""Frames of the Craftax world for people to look at (``priml/baselines/craftax/game/render/pixels.py``).

The reference blits sprites with pygame, one worker per call. Here a frame is a
tensor program over the whole batch, on whatever device holds the game state:

* every sprite lives in one RGBA atlas ``[N, P, P, 4]``;
* each layer -- terrain, items, creatures and projectiles, the player -- is a
  ``[E, rows, cols]`` map of atlas indices (``-1`` where the layer is empty);
  one gather turns it into pixels and one blend lays it over the frame;
* shading multiplies last: unseen tiles go black (the observation's visibility
  rule, :func:`~priml_b200.baselines.craftax.game.observation.visible_tiles`), the
  surface fades toward night blue after dark, sleep halves the brightness.

The frame is the player's own 9 x 11 view, the window the policy reads. No
graphics library is involved. Sprites are the game's upstream PNGs (MIT
licensed, named as upstream names them) read from ``sprite_dir`` when it holds
them; there is no download, and a missing file gets a generated stand-in: a flat
tile of a colour derived from the sprite's name, and for creatures, items and
the player a disc over a transparent corner, so layers stay distinguishable.
"""

from __future__ import annotations

import hashlib
from pathlib import Path

import torch
import torch.nn.functional as F
from torch import Tensor

from priml_b200.baselines.craftax.game import constants as C
from priml_b200.baselines.craftax.game.observation import local_view, visible_tiles
from priml_b200.baselines.craftax.game.state import GameState

__all__ = ["BLOCK_SPRITES", "ITEM_SPRITES", "PixelRenderer"]

# Upstream sprite file names, one per enum value ("" = flat colour, no art).
BLOCK_SPRITES: tuple[str, ...] = (
    "debug_tile.png", "", "grass.png", "water.png", "stone.png", "tree.png", "wood.png", "path.png", "coal.png",
    "iron.png", "diamond.png", "table.png", "furnace.png", "sand.png", "lava.png", "plant_on_grass.png",
    "ripe_plant_on_grass.png", "wall2.png", "", "wall_moss.png", "stalagmite.png", "sapphire.png", "ruby.png",
    "chest.png", "fountain.png", "fire_grass.png", "ice_grass.png", "gravel.png", "fire_tree.png", "ice_shrub.png",
    "enchantment_table_fire.png", "enchantment_table_ice.png", "necromancer.png", "grave.png", "grave2.png",
    "grave3.png", "necromancer_vulnerable.png",
)  # fmt: skip
ITEM_SPRITES: tuple[str, ...] = ("", "torch_in_inventory.png", "ladder_down.png", "ladder_up.png",
                                 "ladder_down_blocked.png")  # fmt: skip
PLAYER_SPRITES: tuple[str, ...] = ("player-left.png", "player-right.png", "player-up.png", "player-down.png",
                                   "player-sleep.png")  # fmt: skip
PASSIVE_SPRITES: tuple[str, ...] = ("cow.png", "bat.png", "snail.png")
MELEE_SPRITES: tuple[str, ...] = ("zombie.png", "gnome_warrior.png", "orc_soldier.png", "lizard.png", "knight.png",
                                  "troll.png", "pigman.png", "frost_troll.png")  # fmt: skip
RANGED_SPRITES: tuple[str, ...] = ("skeleton.png", "gnome_archer.png", "orc_mage.png", "kobold.png",
                                   "knight_archer.png", "deep_thing.png", "fire_elemental.png",
                                   "ice_elemental.png")  # fmt: skip
PROJECTILE_SPRITES: tuple[str, ...] = ("arrow-up.png", "dagger.png", "fireball.png", "iceball.png", "arrow-up.png",
                                       "slimeball.png", "fireball.png", "iceball.png")  # fmt: skip
SHOT_SPRITES: tuple[str, ...] = ("arrow-up.png", "fireball.png", "iceball.png")  # the player's arrow, fire, ice

OUT_OF_BOUNDS_COLOR = (128, 128, 128)
DARKNESS_COLOR = (0, 0, 0)
NIGHT_COLOR = (0, 16, 64)


def _stand_in(name: str, p: int, opaque: bool) -> Tensor:
    """A generated ``[P, P, 4]`` sprite: a colour from the name's digest, a darker rim; a disc unless opaque."""
    h = hashlib.sha256(name.encode()).digest()
    rgb = torch.tensor([40 + h[0] % 200, 40 + h[1] % 200, 40 + h[2] % 200], dtype=torch.float32) / 255.0
    ys, xs = torch.meshgrid(torch.arange(p, dtype=torch.float32), torch.arange(p, dtype=torch.float32), indexing="ij")
    edge = torch.minimum(torch.minimum(ys, xs), torch.minimum(p - 1 - ys, p - 1 - xs))
    shade = torch.where(edge < max(1, p // 16), 0.6, 1.0)
    img = torch.empty(p, p, 4)
    img[..., :3] = rgb * shade[..., None]
    if opaque:
        img[..., 3] = 1.0
    else:
        r = ((ys - (p - 1) / 2) ** 2 + (xs - (p - 1) / 2) ** 2).sqrt()
        img[..., 3] = (r <= p * 0.4).float()
    return img


def _load_png(path: Path, p: int) -> Tensor:
    from torchvision.io import ImageReadMode, decode_png, read_file

    img = decode_png(read_file(str(path)), ImageReadMode.RGB_ALPHA).float() / 255.0  # [4, h, w]
    img = F.interpolate(img[None], size=(p, p), mode="nearest")[0]
    return img.permute(1, 2, 0).contiguous()


class PixelRenderer:
    """``render(state) -> [E, rows * P, cols * P, 3]`` uint8 frames of every world in the batch."""

    def __init__(self, *, block_pixels: int = 16, sprite_dir: str | Path | None = None,
                 device: torch.device | str | None = None) -> None:  # fmt: skip
        if block_pixels <= 0:
            raise ValueError("block_pixels must be positive")
        self.block_pixels = p = block_pixels
        self.sprite_dir = Path(sprite_dir) if sprite_dir is not None else None
        names: list[str] = []
        index: dict[str, int] = {}

        def add(name: str, opaque: bool) -> int:
            if not name:
                return -1
            if name not in index:
                index[name] = len(names)
                names.append(name)
                self._opaque.append(opaque)
            return index[name]

        self._opaque: list[bool] = []
        blocks = [add(n, True) for n in BLOCK_SPRITES]
        # flat colours as one-colour opaque tiles
        flat = {}
        for enum, colour in ((C.BlockType.OUT_OF_BOUNDS, OUT_OF_BOUNDS_COLOR), (C.BlockType.DARKNESS, DARKNESS_COLOR)):
            flat[len(names)] = colour
            blocks[int(enum)] = add(f"<flat {int(enum)}>", True)
        self.found: list[str] = []
        tables = {
            "items": [add(n, False) for n in ITEM_SPRITES],
            "player": [add(n, False) for n in PLAYER_SPRITES],
            "passive": [add(n, False) for n in PASSIVE_SPRITES],
            "melee": [add(n, False) for n in MELEE_SPRITES],
            "ranged": [add(n, False) for n in RANGED_SPRITES],
            "projectile": [add(n, False) for n in PROJECTILE_SPRITES],
            "shot": [add(n, False) for n in SHOT_SPRITES],
        }
        atlas = []
        for i, name in enumerate(names):
            if i in flat:
                tile = torch.ones(p, p, 4)
                tile[..., :3] = torch.tensor(flat[i], dtype=torch.float32) / 255.0
            elif self.sprite_dir is not None and (self.sprite_dir / name).exists():
                tile = _load_png(self.sprite_dir / name, p)
                self.found.append(name)
            else:
                tile = _stand_in(name, p, self._opaque[i])
            atlas.append(tile)
        self.device = torch.device(device) if device is not None else torch.device("cpu")
        self.atlas = torch.stack(atlas).to(self.device)  # [N, P, P, 4]
        self.tables = {k: torch.tensor(v, dtype=torch.long, device=self.device) for k, v in tables.items()}
        self.tables["blocks"] = torch.tensor(blocks, dtype=torch.long, device=self.device)

    # ------------------------------------------------------------------ layers
    def _pixels(self, idx: Tensor) -> Tensor:
        """``[E, r, c]`` atlas indices -> ``[E, r * P, c * P, 4]`` RGBA (alpha 0 where the index is -1)."""
        e, r, c = idx.shape
        p = self.block_pixels
        tiles = self.atlas[idx.clamp(min=0)]  # [E, r, c, P, P, 4]
        tiles = tiles * (idx >= 0)[..., None, None, None]
        return tiles.permute(0, 1, 3, 2, 4, 5).reshape(e, r * p, c * p, 4)

    @staticmethod
    def _over(frame: Tensor, layer: Tensor) -> Tensor:
        a = layer[..., 3:]
        return frame * (1 - a) + layer[..., :3] * a

    def _creature_layer(self, s: GameState, creatures, sprite_idx: Tensor, view: tuple[int, int]) -> Tensor:  # noqa: ANN001
        """Atlas indices of one creature class's live slots inside the view (``sprite_idx``: ``[E, S]``)."""
        vr, vc = view
        e = s.num_envs
        out = torch.full((e, vr * vc + 1), -1, dtype=torch.long, device=s.device)
        corner = s.position - torch.tensor([vr // 2, vc // 2], device=s.device)
        local = creatures.position - corner[:, None, :]  # [E, S, 2]
        inside = creatures.mask & (local[..., 0] >= 0) & (local[..., 0] < vr) & (local[..., 1] >= 0) & (local[..., 1] < vc)
        cell = torch.where(inside, local[..., 0] * vc + local[..., 1], vr * vc)  # outside -> the spare slot
        out.scatter_(1, cell, torch.where(inside, sprite_idx, -1))
        return out[:, :-1].view(e, vr, vc)

    # ------------------------------------------------------------------ frame
    @torch.no_grad()
    def render(self, s: GameState, view: tuple[int, int] = C.OBS_DIM) -> Tensor:
        dev = s.device
        t = {k: v.to(dev) for k, v in self.tables.items()}
        atlas = self.atlas.to(dev)
        self.atlas, self.tables = atlas, t
        vr, vc = view
        e = s.num_envs
        env = torch.arange(e, device=dev)
        blocks, items = local_view(s, view)
        last = s.level == C.LEVELS - 1
        vulnerable = last & ~s.melee.mask.any(-1) & ~s.ranged.mask.any(-1) & (s.boss_wait <= 0)
        blocks = torch.where((blocks == int(C.BlockType.NECROMANCER)) & vulnerable[:, None, None],
                             int(C.BlockType.NECROMANCER_VULNERABLE), blocks)  # fmt: skip
        cleared = s.kills[env, s.level] >= C.MONSTERS_KILLED_TO_CLEAR_LEVEL
        items = torch.where((items == int(C.ItemType.LADDER_DOWN)) & ~cleared[:, None, None],
                            int(C.ItemType.LADDER_DOWN_BLOCKED), items)  # fmt: skip

        frame = self._pixels(t["blocks"][blocks])[..., :3]
        frame = self._over(frame, self._pixels(t["items"][items]))

        species = C.device_table("species", dev, C.FLOOR_SPECIES)[s.level]  # [E, 3] (passive, melee, ranged)
        slots = lambda table, ids, n: table[ids.clamp(0, table.numel() - 1)][:, None].expand(-1, n)  # noqa: E731
        for creatures, sprite in (
            (s.passive, slots(t["passive"], species[:, 0], s.passive.mask.shape[1])),
            (s.melee, slots(t["melee"], species[:, 1], s.melee.mask.shape[1])),
            (s.ranged, slots(t["ranged"], species[:, 2], s.ranged.mask.shape[1])),
            (s.projectiles, slots(t["projectile"], species[:, 2], s.projectiles.mask.shape[1])),
            (s.shots, t["shot"][s.shots.cooldown.long().clamp(0, t["shot"].numel() - 1)]),
        ):
            frame = self._over(frame, self._pixels(self._creature_layer(s, creatures, sprite, view)))

        facing = torch.where(s.sleeping, len(PLAYER_SPRITES) - 1, (s.direction - 1).clamp(0, 3))
        player = torch.full((e, vr, vc), -1, dtype=torch.long, device=dev)
        player[:, vr // 2, vc // 2] = t["player"][facing]
        frame = self._over(frame, self._pixels(player))

        p = self.block_pixels
        seen = visible_tiles(s, items, view).float()
        frame = frame * seen.repeat_interleave(p, 1).repeat_interleave(p, 2)[..., None]
        daylight = torch.where(s.level > 0, torch.ones_like(s.light), s.light.float()).clamp(0, 1)
        night = torch.tensor(NIGHT_COLOR, dtype=frame.dtype, device=dev) / 255.0
        a = (1 - daylight)[:, None, None, None]
        frame = frame * (1 - a) + night * a
        frame = torch.where(s.sleeping[:, None, None, None], frame * 0.5, frame)
        return (frame.clamp(0, 1) * 255).round().to(torch.uint8)

    @staticmethod
    def write_png(frame: Tensor, path: str | Path) -> None:
        """Save one ``[H, W, 3]`` uint8 frame as a PNG file."""
        from torchvision.io import write_png

        write_png(frame.detach().cpu().permute(2, 0, 1).contiguous(), str(path))
