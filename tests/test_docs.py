"""The README's commands name modules and configs that exist, and the
documentation does not point at files that are missing."""

import importlib
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_readme_modules_and_configs_exist():
    text = (ROOT / "README.md").read_text(encoding="utf-8")
    modules = set(re.findall(r"python -m (graspo_b200(?:\.[a-z_0-9]+)*)", text))
    assert "graspo_b200.analysis.profile" in modules
    for mod in modules:
        importlib.import_module(mod)
    for cfg in re.findall(r"(configs/[a-z0-9_]+\.yaml)", text):
        assert (ROOT / cfg).exists(), cfg


def test_design_and_profiles_reference_existing_files():
    design = (ROOT / "DESIGN.md").read_text(encoding="utf-8")
    for path in set(re.findall(r"`((?:csrc|graspo_b200|tests|configs|profiles)/[A-Za-z0-9_./]+\.(?:cu|cuh|py|cpp|yaml|md))`",
                               design)):
        assert (ROOT / path).exists(), path
    profiles = sorted((ROOT / "profiles").glob("*.md"))
    assert len(profiles) >= 5
    for p in profiles:
        assert "ncu" in p.read_text(encoding="utf-8"), p.name  # every summary states how it was captured
