"""SUR support selection (host side): units and allocation against the
reference's outputs on seeded prompts (tests/golden/selection.json, made by
tests/golden/make_selection_golden.py) and the reference's own unit tests
(tests/test_semantic_units.py of the reference), restated."""

import json
import math
import os
import re

import pytest

from conftest import GOLDEN

from budgeted_kv_cache_repair_b200.selection import (best_forward_causal_window, score_semantic_units,
                                                      select_semantic_unit_support, semantic_char_units,
                                                      semantic_unit_token_ranges)


class CharTokenizer:
    """One token per character, exact offsets (the reference tests' tokenizer)."""

    def __call__(self, text, *, add_special_tokens=False, return_offsets_mapping=False):
        assert add_special_tokens is False
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


def _cases():
    with open(os.path.join(GOLDEN, "selection.json")) as fh:
        return json.load(fh)["cases"]


def _rows(units):
    return [[u["start"], u["end"], str(u["container_id"]), u["container_kind"], u["boundary_kind"]] for u in units]


@pytest.mark.parametrize("index", range(len(_cases())))
def test_units_and_allocation_match_reference(index):
    case = _cases()[index]
    text = case["text"]
    tokenizer = CharTokenizer() if case["tokenizer"] == "char" else WordTokenizer()
    assert _rows(semantic_char_units(text)) == case["char_units"]
    units = semantic_unit_token_ranges(tokenizer=tokenizer, text=text, expected_token_ids=tokenizer(text)["input_ids"],
                                       suffix_start=case["suffix_start"], token_end=case["token_end"])
    assert _rows(units) == case["units"]
    for alloc in case["allocations"]:
        support, meta = select_semantic_unit_support(units=units, token_scores=case["scores"],
                                                     budget_tokens=alloc["budget"])
        assert support == alloc["support"]
        assert [u["unit_score"] for u in meta["units"]] == alloc["unit_scores"]
        assert [{k: s[k] for k in ("rank", "unit_index", "selection_kind", "selected_start", "selected_end")}
                for s in meta["selections"]] == alloc["selections"]


def _unit(start, end, container=0):
    return {"start": start, "end": end, "container_id": container, "container_kind": "ordinary_text",
            "boundary_kind": "generic_sentence_or_paragraph"}


@pytest.mark.parametrize("peak, expected", [(None, (0, 5)), (2, (2, 7)), (10, (10, 15))])
def test_partial_window_tracks_peak_without_tail_bias(peak, expected):
    scores = [0.0] * 20 if peak is None else [-100.0] * 20
    if peak is not None:
        scores[peak] = 0.0
    window = best_forward_causal_window(start=0, end=20, width=5, token_scores=scores)
    assert (window["start"], window["end"]) == expected
    assert window["decay_tokens"] == 16.0


@pytest.mark.parametrize("width", [0, -1, 21])
def test_partial_window_rejects_invalid_width(width):
    with pytest.raises(ValueError, match="partial-window width"):
        best_forward_causal_window(start=0, end=20, width=width, token_scores=[0.0] * 20)


def test_units_use_canonical_offsets_and_clip_at_token_end():
    tokenizer = CharTokenizer()
    text = "Alpha support sentence.\n\nQuestion: Where?"
    end = text.index("\n\nQuestion:")
    units = semantic_unit_token_ranges(tokenizer=tokenizer, text=text, expected_token_ids=tokenizer(text)["input_ids"],
                                       suffix_start=0, token_end=end)
    support, _ = select_semantic_unit_support(units=units, token_scores=[float(i) for i in range(end)],
                                              budget_tokens=5)
    assert [(u["start"], u["end"]) for u in units] == [(0, end)]
    assert support == list(range(end - 5, end))


def test_units_reject_tokenizer_identity_drift():
    with pytest.raises(RuntimeError, match="tokenizer identity drift"):
        semantic_unit_token_ranges(tokenizer=CharTokenizer(), text="A sentence.", expected_token_ids=[0],
                                   suffix_start=0)


def test_long_units_use_balanced_chunks():
    units = semantic_unit_token_ranges(tokenizer=CharTokenizer(), text="A" * 257,
                                       expected_token_ids=[ord("A")] * 257, suffix_start=0)
    assert [(u["start"], u["end"]) for u in units] == [(0, 86), (86, 172), (172, 257)]


def test_structured_units_keep_tool_and_json_containers():
    text = '<tool_result>{"place": "Oslo."}</tool_result>\n\nMetadata: {"count": 2}\n'
    units = semantic_char_units(text)
    structured = [(u["boundary_kind"], text[u["start"]:u["end"]]) for u in units
                  if u["boundary_kind"] != "generic_sentence_or_paragraph"]
    assert structured == [("tool_container", '<tool_result>{"place": "Oslo."}</tool_result>'),
                          ("json_container", '{"count": 2}')]
    assert "".join(text[u["start"]:u["end"]] for u in units) == text


def test_unit_ranking_uses_top_four_not_all_token_mean():
    units = [_unit(0, 8), _unit(8, 16)]
    scores = [4.0] * 4 + [-100.0] * 4 + [3.0] * 8
    ranked = score_semantic_units(units=units, token_scores=scores)
    support, meta = select_semantic_unit_support(units=units, token_scores=scores, budget_tokens=8)
    assert [u["unit_score"] for u in ranked] == [4.0, 3.0]
    assert support == list(range(8))
    assert meta["selections"][0]["selection_kind"] == "complete_unit"
    assert meta["kv_probe_token_calls"] == meta["planning_expansion_token_calls"] == 0


def test_unit_ties_prefer_earlier_position_and_fill_final_window():
    support, meta = select_semantic_unit_support(units=[_unit(4, 12), _unit(12, 20)], token_scores=[0.0] * 20,
                                                 budget_tokens=11)
    assert support == list(range(4, 15))
    assert [s["selection_kind"] for s in meta["selections"]] == ["complete_unit", "partial_forward_causal_window"]
    assert meta["budget_tokens"] == 11


@pytest.mark.parametrize("bad", [math.inf, -math.inf, math.nan])
def test_unit_scoring_rejects_nonfinite_values(bad):
    with pytest.raises(RuntimeError, match="invalid semantic unit token scores"):
        score_semantic_units(units=[_unit(0, 2)], token_scores=[1.0, bad])


def test_scoring_rejects_cpu_tables_without_fallback():
    import torch

    from budgeted_kv_cache_repair_b200.selection import dense_query_relevance_scores

    table = torch.nn.Embedding(4, 8)
    with pytest.raises(ValueError, match="CUDA"):
        dense_query_relevance_scores(model=type("M", (), {"get_input_embeddings": lambda self: table})(),
                                     edited_input_ids=torch.tensor([[0, 1]]), query_token_ids=[1])
