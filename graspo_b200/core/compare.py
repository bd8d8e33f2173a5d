"""Recursive structured comparison of a predicted dict against a target dict.

The score is ``check / total`` where ``total`` counts everything the target
asks for and ``check`` credits what the prediction got right.  The counting
rules are the reference's (src/graspo/core/compare.py:67-211) because rewards
must be numerically identical across frameworks:

* ``total``: +1 per (sub)dict, +1 per key, +1 per scalar value, +1 per list key,
  each list element (dicts recursively, scalars +1), +1 for order when
  ``check_list_order``.
* ``check``: +1 per target key present, +1 if the prediction has no extra keys,
  recursive credit for sub-dicts, best-matching credit per target list element,
  +1 when the prediction's list holds no foreign element (+1 more when it also
  equals the target in order and every element matched fully), and a leaf score
  (1 for equality, ``1/(1+|a-b|)`` for numbers, bools only equal bools).
* ``base_*``: the same with numeric leaves removed on both sides; ``all_right``
  means every non-numeric item matched.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any


@dataclass(slots=True)
class CompareResult:
    dcs: float = 0.0
    total_score: int = 0
    check_score: float = 0.0
    base_dcs: float = 0.0
    base_total: int = 0
    base_check: float = 0.0

    @property
    def all_right(self) -> bool:
        return self.base_total > 0 and self.base_check == self.base_total


def _is_number(value: Any) -> bool:
    return isinstance(value, (int, float)) and not isinstance(value, bool)


def strip_numeric(value: Any) -> Any:
    """Drop numeric leaves (and dicts left empty by that) from a JSON value.

    A bare number becomes ``None``; lists keep their length (elements are
    stripped individually).
    """
    if isinstance(value, dict):
        out: dict[str, Any] = {}
        for key, item in value.items():
            kept = strip_numeric(item)
            if kept is None or (isinstance(kept, dict) and not kept):
                continue
            out[key] = kept
        return out
    if isinstance(value, list):
        return [strip_numeric(item) for item in value]
    return None if _is_number(value) else value


def count_target_score(target: dict[str, Any], check_list_order: bool, total: int = 0) -> int:
    """Denominator: how many scoring units ``target`` contains."""
    total += 1  # the dict itself
    for value in target.values():
        total += 1  # the key
        if isinstance(value, dict):
            total = count_target_score(value, check_list_order, total)
        elif isinstance(value, list):
            total += 1  # the list as a whole
            for element in value:
                if isinstance(element, dict):
                    total = count_target_score(element, check_list_order, total)
                else:
                    total += 1
            if check_list_order:
                total += 1
        else:
            total += 1
    return total


def leaf_compare_score(checked: Any, target: Any) -> float:
    if isinstance(checked, bool) or isinstance(target, bool):
        same_kind = type(checked) is bool and type(target) is bool
        return 1.0 if same_kind and checked == target else 0.0
    if _is_number(checked) and _is_number(target):
        a, b = float(checked), float(target)
        if math.isfinite(a) and math.isfinite(b):
            return 1.0 / (1.0 + abs(a - b))
        return 1.0 if checked == target else 0.0
    return 1.0 if checked == target else 0.0


def _best_element_match(
    candidates: list[Any], wanted: Any, check_list_order: bool
) -> tuple[float, int]:
    """Credit for one target list element: (check, total) of its best match."""
    if not isinstance(wanted, dict):
        return (1.0, 1) if wanted in candidates else (0.0, 0)
    best_check, best_total = 0.0, 1
    for candidate in candidates:
        if not isinstance(candidate, dict):
            continue
        res = dict_compare_score(candidate, wanted, check_list_order)
        if res.total_score <= 0:
            continue
        # The initial (0, 1) placeholder is always replaced by the first
        # scoreable candidate; afterwards only a strictly better ratio wins.
        placeholder = best_check == 0.0 and best_total == 1
        if placeholder or res.check_score / res.total_score > best_check / best_total:
            best_check, best_total = res.check_score, res.total_score
    return best_check, best_total


def count_check_score(
    checked: dict[str, Any],
    target: dict[str, Any],
    check_list_order: bool,
    score: float = 0.0,
) -> float:
    """Numerator: credit earned by ``checked`` against ``target``."""
    score += sum(1 for key in target if key in checked)
    if all(key in target for key in checked):
        score += 1
    for key, want in target.items():
        if key not in checked:
            continue
        got = checked[key]
        if isinstance(got, dict) and isinstance(want, dict):
            score = count_check_score(got, want, check_list_order, score)
        elif isinstance(got, list) and isinstance(want, list):
            complete = True
            for element in want:
                elem_check, elem_total = _best_element_match(got, element, check_list_order)
                score += elem_check
                if elem_total == 0 or elem_check < elem_total:
                    complete = False
            if all(element in want for element in got):
                score += 1
                if complete and check_list_order and got == want:
                    score += 1
        else:
            score += leaf_compare_score(got, want)
    return score


def dict_compare_score(
    checked: dict[str, Any],
    target: dict[str, Any],
    check_list_order: bool = False,
) -> CompareResult:
    total = count_target_score(target, check_list_order)
    check = count_check_score(checked, target, check_list_order)
    base_checked = strip_numeric(checked)
    base_target = strip_numeric(target)
    base_total, base_check = 0, 0.0
    if isinstance(base_checked, dict) and isinstance(base_target, dict):
        base_total = count_target_score(base_target, check_list_order)
        base_check = count_check_score(base_checked, base_target, check_list_order)
    return CompareResult(
        dcs=check / total if total else 0.0,
        total_score=total,
        check_score=check,
        base_dcs=base_check / base_total if base_total else 0.0,
        base_total=base_total,
        base_check=base_check,
    )
