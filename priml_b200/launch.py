"""Command-line launcher (``priml/launch.py:85-301``).

    python -m priml_b200 pkg.module.factory [--override PATH=VALUE]... [--loglevel LEVEL] [job args...]

Resolves ``factory()`` to a config tree, applies overrides (dotted paths,
JSON-parsed values cast to each field's type), stamps run identity and the
factory's docstring, logs the full config, makes the job and runs it with
SIGTERM turned into ``KeyboardInterrupt`` so ``finally`` blocks (tracker
flush, checkpoint) run. Arguments it does not own go to ``job.run``.
Under ``torch.distributed.run`` each rank runs this same entry point.
"""

from __future__ import annotations

import argparse
import contextlib
import importlib
import inspect
import logging
import signal
import sys
import time
from collections.abc import Iterator
from typing import Any

from priml_b200.config import apply_overrides, resolve_config
from priml_b200.logger import setup_logging

__all__ = ["main"]

log = logging.getLogger(__name__)


def _parse_args(argv: list[str] | None = None) -> tuple[argparse.Namespace, list[str]]:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter, add_help=False)
    p.add_argument("config", type=str, help="dotted path of a function returning a Makeable job config")
    p.add_argument("--loglevel", default="INFO", choices=["DEBUG", "INFO", "WARNING", "ERROR", "CRITICAL"])
    p.add_argument("--override", action="append", default=[], metavar="PATH=VALUE")
    return p.parse_known_args(argv)


@contextlib.contextmanager
def _graceful_sigterm() -> Iterator[None]:
    def handler(signum: int, frame: Any) -> None:
        del signum, frame
        raise KeyboardInterrupt("SIGTERM")

    old = signal.signal(signal.SIGTERM, handler)
    try:
        yield
    finally:
        signal.signal(signal.SIGTERM, old)


def _derive_study_name(module_name: str) -> str:
    parts = module_name.split(".")
    try:
        i = parts.index("experimental")
        between = parts[i + 1 : parts.index("experiments")]
    except ValueError:
        return ""
    return "/".join(between) + "/" if between else ""


def _log_hardware() -> None:
    try:
        import torch

        if torch.cuda.is_available():
            p = torch.cuda.get_device_properties(0)
            log.info("device: %s, %d SMs, %.0f GB", p.name, p.multi_processor_count, p.total_memory / 1e9)
    except Exception:  # noqa: BLE001
        pass


def main(argv: list[str] | None = None) -> int:
    t0 = time.perf_counter()
    args, rest = _parse_args(argv)
    setup_logging(args.loglevel)
    _log_hardware()
    module_name, fn_name = args.config.rsplit(".", 1)
    config = resolve_config(args.config)
    apply_overrides(config, args.override)
    fn = getattr(importlib.import_module(module_name), fn_name)
    doc = inspect.getdoc(fn) or ""
    if hasattr(config, "experiment_name") and not getattr(config, "experiment_name"):
        config.experiment_name = fn_name
    if hasattr(config, "study_name") and not getattr(config, "study_name"):
        config.study_name = _derive_study_name(module_name)
    if hasattr(config, "doc") and doc and not getattr(config, "doc"):
        config.doc = doc
    log.info("experiment %s docstring:\n%s", args.config, doc or "(none)")
    pf = getattr(config, "pformat", None)
    log.info("experiment config %s:\n%s", args.config, pf(finalize=True, hide_default_values=False) if callable(pf) else repr(config))
    job = config.make()
    if not hasattr(job, "run"):
        raise TypeError(f"{args.config!r} made {type(job).__name__}, which has no run()")
    with _graceful_sigterm():
        job.run(*rest)
    log.info("Total program time: %.1fs", time.perf_counter() - t0)
    return 0


if __name__ == "__main__":
    sys.exit(main())
