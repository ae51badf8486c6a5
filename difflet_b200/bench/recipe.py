"""Bench recipes: named sets of the engine's own ``generate`` flags.

Behaviour of the reference's recipes (difflet/bench/recipe.py:1-60, recipes.yaml): a recipe's
``args`` keys are ``generate`` flag names without the leading dashes (``true`` = bare switch,
``false`` = switch left out, anything else = ``--flag value``); ``extends`` inherits another recipe
and overrides it; ``env.force`` is set in the launched engine's environment whatever the caller
has, ``env.default`` only where the caller has not; names starting with ``_`` are abstract.  The
flags the harness owns (output, cache / work directories, requests, force) may not be set by a
recipe.  Recipes are validated by the real ``generate`` parser, so a new CLI flag works in a recipe
the day it lands and a misspelt one is refused before anything is launched.
"""

from __future__ import annotations

import contextlib
import hashlib
import io
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Mapping

RECIPES_FILE = Path(__file__).with_name("recipes.yaml")
SELF_MANAGED = frozenset({"output", "cache-dir", "work-dir", "keep-work-dir", "requests", "force"})
REQUIRED = ("model-id", "prompt")
TOP_LEVEL = frozenset({"description", "extends", "args", "env"})
ENV_LAYERS = frozenset({"force", "default"})


class RecipeError(ValueError):
    """A recipe, suite variant or override that the harness refuses to run."""


@dataclass(frozen=True)
class Recipe:
    name: str
    args: dict[str, Any]
    env_force: dict[str, str] = field(default_factory=dict)
    env_default: dict[str, str] = field(default_factory=dict)
    description: str = ""

    def with_args(self, extra: Mapping[str, Any] | None, name: str | None = None) -> "Recipe":
        return Recipe(name or self.name, merge_args(self.args, extra or {}), dict(self.env_force),
                      dict(self.env_default), self.description)

    def argv(self) -> list[str]:
        return to_argv(self.args)

    def env(self, base: Mapping[str, str]) -> dict[str, str]:
        """The launched engine's environment: ``base`` + defaults it lacks + forced values."""
        out = dict(base)
        for k, v in self.env_default.items():
            out.setdefault(k, str(v))
        out.update({k: str(v) for k, v in self.env_force.items()})
        return out


def merge_args(low: Mapping[str, Any], high: Mapping[str, Any]) -> dict[str, Any]:
    out = dict(low)
    out.update(high)
    return out


def to_argv(args: Mapping[str, Any]) -> list[str]:
    argv = []
    for k, v in args.items():
        if v is False or v is None:
            continue
        argv.append(f"--{k}")
        if v is not True:
            argv.append(str(v))
    return argv


def _load_yaml(path: Path) -> dict:
    import yaml

    doc = yaml.safe_load(Path(path).read_text()) or {}
    if not isinstance(doc, dict):
        raise RecipeError(f"{path}: a recipe file is a mapping of recipe names")
    return doc


def resolve(name: str, table: Mapping[str, Any], _seen: tuple = ()) -> Recipe:
    """``name`` with its ``extends`` chain merged (not yet validated against the CLI)."""
    if name in _seen:
        raise RecipeError(f"recipe cycle: {' -> '.join(_seen + (name,))}")
    if name not in table:
        raise RecipeError(f"unknown recipe {name!r}")
    body = table[name] or {}
    bad = set(body) - TOP_LEVEL
    if bad:
        raise RecipeError(f"recipe {name!r}: unknown keys {sorted(bad)}")
    env = body.get("env") or {}
    if set(env) - ENV_LAYERS:
        raise RecipeError(f"recipe {name!r}: env layers are {sorted(ENV_LAYERS)}")
    base = resolve(body["extends"], table, _seen + (name,)) if body.get("extends") else Recipe(name, {})
    force = dict(base.env_force)
    force.update({k: str(v) for k, v in (env.get("force") or {}).items()})
    default = dict(base.env_default)
    default.update({k: str(v) for k, v in (env.get("default") or {}).items()})
    return Recipe(name, merge_args(base.args, body.get("args") or {}), force, default,
                  body.get("description", base.description))


def load_recipes(path: Path | str | None = None) -> dict[str, Recipe]:
    """Every concrete (non-``_``) recipe of the file, resolved."""
    table = _load_yaml(Path(path) if path else RECIPES_FILE)
    return {n: resolve(n, table) for n in table if not n.startswith("_")}


def validate(recipe: Recipe) -> Recipe:
    """Refuse harness-owned flags, missing required flags and anything ``generate`` rejects."""
    owned = SELF_MANAGED & set(recipe.args)
    if owned:
        raise RecipeError(f"recipe {recipe.name!r} sets flags the harness owns: {sorted(owned)}")
    missing = [k for k in REQUIRED if recipe.args.get(k) in (None, False)]
    if missing:
        raise RecipeError(f"recipe {recipe.name!r} lacks required flags {missing}")
    from difflet_b200.cli.main import build_parser

    parser = build_parser()
    argv = ["generate", *recipe.argv(), "--output", "/dev/null"]
    try:
        with contextlib.redirect_stderr(io.StringIO()):
            parser.parse_args(argv)
    except SystemExit as exc:
        raise RecipeError(f"recipe {recipe.name!r}: generate rejects {recipe.argv()}") from exc
    return recipe


def file_sha256(path: Path | str | None = None) -> str:
    return hashlib.sha256(Path(path or RECIPES_FILE).read_bytes()).hexdigest()


__all__ = ["RECIPES_FILE", "Recipe", "RecipeError", "file_sha256", "load_recipes", "merge_args", "resolve",
           "to_argv", "validate"]
