"""Generate ``selection.json``: the reference's SUR units and allocations on
seeded synthetic prompts.

    python tests/golden/make_selection_golden.py --reference <checkout of yh0903/budgeted-kv-cache-repair>

Runs the reference's ``semantic_char_units``, ``semantic_unit_token_ranges``
and ``select_semantic_unit_support`` (semantic_units.py:214-576) on prompts
assembled here from a small word list plus chat-template blocks, tool blocks,
inline JSON, blank lines and long unpunctuated runs, under two tokenizers with
offset mappings (one token per character; one token per whitespace-separated
word), with seeded token scores and several budgets. Nothing at test time
reads the reference; ``tests/test_selection.py`` reads only the JSON.
"""

from __future__ import annotations

import argparse
import json
import os
import random
import re
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
WORDS = ["alpha", "beta", "gamma", "delta", "Omega", "river", "stone", "lamp", "quiet", "North", "7", "x"]


class CharTokenizer:
    def __call__(self, text, *, add_special_tokens=False, return_offsets_mapping=False):
        out = {"input_ids": [ord(c) for c in text]}
        if return_offsets_mapping:
            out["offset_mapping"] = [(i, i + 1) for i in range(len(text))]
        return out


class WordTokenizer:
    def __call__(self, text, *, add_special_tokens=False, return_offsets_mapping=False):
        spans = [(m.start(), m.end()) for m in re.finditer(r"\S+", text)]
        out = {"input_ids": [sum(ord(c) for c in text[a:b]) % 1000 for a, b in spans]}
        if return_offsets_mapping:
            out["offset_mapping"] = spans
        return out


def sentence(rng, n):
    words = [rng.choice(WORDS) for _ in range(n)]
    return " ".join(words) + rng.choice([".", "!", "?", ".)", "."])


def prompt(rng):
    parts = []
    for _ in range(rng.randint(3, 9)):
        kind = rng.random()
        if kind < 0.45:
            parts.append(" ".join(sentence(rng, rng.randint(1, 14)) for _ in range(rng.randint(1, 4))))
        elif kind < 0.55:
            parts.append("<|im_start|>user\n" + sentence(rng, rng.randint(2, 9)) + "<|im_end|>")
        elif kind < 0.65:
            parts.append('<tool_result>{"place": "' + rng.choice(WORDS) + '.", "n": ' + str(rng.randint(0, 99))
                         + "}</tool_result>")
        elif kind < 0.75:
            parts.append("Metadata: {\"count\": " + str(rng.randint(0, 9)) + ", \"tags\": [\"" + rng.choice(WORDS)
                         + "\"]}")
        elif kind < 0.85:
            parts.append(" ".join(rng.choice(WORDS) for _ in range(rng.randint(40, 90))))  # long, no punctuation
        else:
            parts.append(rng.choice(["x.", "Go!", "7?", "a b."]))  # short units
    sep = [" ", "\n", "\n\n", "\n \n"]
    return "".join(p + rng.choice(sep) for p in parts)


def main():
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--reference", required=True)
    parser.add_argument("--cases", type=int, default=60)
    args = parser.parse_args()
    sys.path.insert(0, os.path.join(args.reference, "src"))
    from kv_cache_repair.semantic_units import (select_semantic_unit_support, semantic_char_units,
                                                semantic_unit_token_ranges)

    rng = random.Random(1234)
    cases = []
    while len(cases) < args.cases:
        text = prompt(rng)
        tok = rng.choice(["char", "word"])
        tokenizer = CharTokenizer() if tok == "char" else WordTokenizer()
        ids = tokenizer(text)["input_ids"]
        if len(ids) < 4:
            continue
        suffix_start = rng.randint(0, len(ids) - 2)
        token_end = None if rng.random() < 0.7 else rng.randint(suffix_start + 1, len(ids))
        units = semantic_unit_token_ranges(tokenizer=tokenizer, text=text, expected_token_ids=ids,
                                           suffix_start=suffix_start, token_end=token_end)
        end = len(ids) if token_end is None else token_end
        scores = [round(rng.gauss(0.0, 1.0), 3) if rng.random() < 0.9 else 0.5 for _ in range(len(ids))]
        allocations = []
        for budget in sorted({1, max(1, (end - suffix_start) // 20), max(1, (end - suffix_start) // 3),
                              end - suffix_start}):
            support, meta = select_semantic_unit_support(units=units, token_scores=scores, budget_tokens=budget)
            allocations.append(dict(budget=budget, support=support,
                                    selections=[{k: s[k] for k in ("rank", "unit_index", "selection_kind",
                                                                   "selected_start", "selected_end")}
                                                for s in meta["selections"]],
                                    unit_scores=[u["unit_score"] for u in meta["units"]]))
        cases.append(dict(text=text, tokenizer=tok, suffix_start=suffix_start, token_end=token_end, scores=scores,
                          char_units=[[u["start"], u["end"], str(u["container_id"]), u["container_kind"],
                                       u["boundary_kind"]] for u in semantic_char_units(text)],
                          units=[[u["start"], u["end"], str(u["container_id"]), u["container_kind"],
                                  u["boundary_kind"]] for u in units],
                          allocations=allocations))
    with open(os.path.join(HERE, "selection.json"), "w") as fh:
        json.dump({"generator": "tests/golden/make_selection_golden.py", "cases": cases}, fh, separators=(",", ":"))
    print(len(cases), "cases")


if __name__ == "__main__":
    main()
