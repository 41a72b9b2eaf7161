"""Support selection for ``select_support`` (SUR V1): semantic units of the
edited prompt, frozen-embedding query relevance on the B200, and the
exact-budget unit allocator.

Follows the reference's rules (semantic_units.py:1-576, scoring.py:11-88,
api.py:83-96) so that the same prompt, query and scores select the same
positions:

* Text units. Chat-template blocks (``<|im_start|>...<|im_end|>``) are
  containers, the text around them ordinary containers (a whitespace-only gap
  joins the container before it). Inside a container, tool/function blocks
  and JSON objects or arrays (a ``[``/``{`` that opens a line or follows
  ``:``, ``=`` or ``>``, and parses as JSON) are kept whole, earliest and then
  longest first, non-overlapping; the remaining text is cut at sentence ends
  and blank lines.
* Token units. Suffix tokens map to the text unit holding their offset
  midpoint; runs of tokens in one text unit form a token unit. Units longer
  than 128 tokens are cut into balanced chunks; units shorter than 8 tokens
  merge with an adjacent unit of the same container (the shorter neighbour,
  the earlier one on ties) and the result is re-chunked, until none is left.
* Scores. Token score = max cosine between its input embedding and the query
  tokens' embeddings, + 0.25 when its id is a query id (one CUDA kernel,
  ``kvr_query_relevance``). Unit score = mean of its top min(4, length) token
  scores.
* Allocation. Units by score (earlier first on ties) are taken whole while
  they fit; the unit that does not fit contributes the contiguous window of
  the remaining width with the largest forward-causal utility (running max of
  exp(score - max) with decay exp(-1/16) per token).
"""

from __future__ import annotations

import json
import math
import re
from typing import Any

import torch

from . import _lib

MIN_UNIT_TOKENS = 8
MAX_UNIT_TOKENS = 128
UNIT_TOP_K = 4
CAUSAL_DECAY_TOKENS = 16.0
EXACT_TOKEN_BOOST = 0.25

# The unit boundaries are part of the selection contract: these three
# patterns are the reference's (semantic_units.py:16-25).
_CHAT = re.compile(r"<\|im_start\|>.*?<\|im_end\|>", flags=re.DOTALL)
_TOOL = re.compile(r"<(?P<tag>tool_call|tool_response|tool_result|function_call|"
                   r"function_response)(?:\s[^>]*)?>.*?</(?P=tag)>", flags=re.DOTALL | re.IGNORECASE)
_SENTENCE_END = re.compile(r"\n[ \t]*\n+|[.!?][\"')\]]*(?:[ \t\r\n]+|(?=[A-Z0-9<]))")
_OPENER = re.compile(r"[\[{]")


def _unit(start, end, container_id, container_kind, boundary_kind, **extra) -> dict[str, Any]:
    row = {"start": int(start), "end": int(end), "container_id": container_id, "container_kind": container_kind,
           "boundary_kind": boundary_kind}
    row.update(extra)
    return row


# ------------------------------------------------------------------ text units
def _json_spans(text: str, lo: int, hi: int) -> list[tuple[int, int]]:
    """JSON objects/arrays inside text[lo:hi] that open a line or follow ':', '=' or '>'."""
    decoder = json.JSONDecoder()
    spans, pos = [], lo
    while pos < hi:
        found = _OPENER.search(text, pos, hi)
        if found is None:
            break
        at = found.start()
        lead = text[text.rfind("\n", lo, at) + 1:at].strip()
        parsed = None
        if not lead or lead.endswith((":", "=", ">")):
            try:
                parsed = decoder.raw_decode(text[at:hi])
            except json.JSONDecodeError:
                parsed = None
        if parsed is not None and isinstance(parsed[0], (dict, list)):
            spans.append((at, at + parsed[1]))
            pos = at + parsed[1]
        else:
            pos = at + 1
    return spans


def _containers(text: str) -> list[dict[str, Any]]:
    """Chat blocks and the ordinary text between them, in order, non-empty."""
    rows: list[dict[str, Any]] = []

    def ordinary(lo: int, hi: int) -> None:
        if rows and not text[lo:hi].strip():
            rows[-1]["end"] = hi  # a whitespace-only gap joins the container before it
        else:
            rows.append(_unit(lo, hi, len(rows), "ordinary_text", None))

    pos = 0
    for block in _CHAT.finditer(text):
        if pos < block.start():
            ordinary(pos, block.start())
        rows.append(_unit(block.start(), block.end(), len(rows), "chat_message", None))
        pos = block.end()
    if pos < len(text):
        ordinary(pos, len(text))
    elif not rows:
        rows.append(_unit(0, len(text), 0, "ordinary_text", None))
    return [r for r in rows if r["end"] > r["start"]]


def _split_container(text: str, box: dict[str, Any]) -> list[dict[str, Any]]:
    """Structured blocks of a container kept whole, the text between them generic."""
    lo, hi = box["start"], box["end"]
    found = [(m.start(), m.end(), "tool_container") for m in _TOOL.finditer(text, lo, hi)]
    found += [(a, b, "json_container") for a, b in _json_spans(text, lo, hi)]
    kept: list[tuple[int, int, str]] = []
    for a, b, kind in sorted(found, key=lambda f: (f[0], f[0] - f[1])):
        if all(not (a < kb and ka < b) for ka, kb, _ in kept):
            kept.append((a, b, kind))
    kept.sort()
    out, pos = [], lo
    for index, (a, b, kind) in enumerate(kept):
        if pos < a:
            out.append(_unit(pos, a, box["container_id"], box["container_kind"], "generic_text"))
        out.append(_unit(a, b, f"{box['container_id']}:structured:{index}", kind, kind))
        pos = b
    if pos < hi:
        out.append(_unit(pos, hi, box["container_id"], box["container_kind"], "generic_text"))
    return [r for r in out if r["end"] > r["start"]]


def _sentences(text: str, lo: int, hi: int) -> list[tuple[int, int]]:
    spans, pos = [], lo
    for cut in _SENTENCE_END.finditer(text, lo, hi):
        if cut.end() > pos:
            spans.append((pos, cut.end()))
        pos = cut.end()
    if pos < hi:
        spans.append((pos, hi))
    return spans or [(lo, hi)]


def semantic_char_units(text: str) -> list[dict[str, Any]]:
    """Character ranges of the text units (semantic_units.py:214-244)."""
    units = []
    for box in _containers(text):
        for part in _split_container(text, box):
            if part["boundary_kind"] == "generic_text":
                spans, kind = _sentences(text, part["start"], part["end"]), "generic_sentence_or_paragraph"
            else:
                spans, kind = [(part["start"], part["end"])], part["boundary_kind"]
            units += [_unit(a, b, part["container_id"], part["container_kind"], kind) for a, b in spans if b > a]
    return units


# ----------------------------------------------------------------- token units
def _chunks(lo: int, hi: int) -> list[tuple[int, int]]:
    """[lo, hi) cut into the fewest near-equal pieces of at most MAX_UNIT_TOKENS."""
    n = hi - lo
    if n <= 0:
        return []
    pieces = -(-n // MAX_UNIT_TOKENS)
    width, wider = divmod(n, pieces)
    out, pos = [], lo
    for k in range(pieces):
        step = width + (k < wider)
        out.append((pos, pos + step))
        pos += step
    return out


def _chunked(unit: dict[str, Any], lo: int, hi: int) -> list[dict[str, Any]]:
    pieces = _chunks(lo, hi)
    return [dict(unit, start=a, end=b, fixed_chunk_index=k, fixed_chunk_count=len(pieces))
            for k, (a, b) in enumerate(pieces)]


def _merge_short(units: list[dict[str, Any]]) -> list[dict[str, Any]]:
    units = list(units)
    while True:
        pick = None
        for i, u in enumerate(units):
            if u["end"] - u["start"] >= MIN_UNIT_TOKENS:
                continue
            options = []
            if i and units[i - 1]["container_id"] == u["container_id"] and units[i - 1]["end"] == u["start"]:
                options.append((units[i - 1]["end"] - units[i - 1]["start"], 0, i - 1))
            if i + 1 < len(units) and units[i + 1]["container_id"] == u["container_id"] \
                    and u["end"] == units[i + 1]["start"]:
                options.append((units[i + 1]["end"] - units[i + 1]["start"], 1, i + 1))
            if options:
                pick = (i, min(options)[2])
                break
        if pick is None:
            return units
        left, right = min(pick), max(pick)
        joined = dict(units[left], boundary_kind="short_unit_merged_within_container")
        units[left:right + 1] = _chunked(joined, units[left]["start"], units[right]["end"])


def semantic_unit_token_ranges(*, tokenizer: Any, text: str, expected_token_ids, suffix_start: int,
                               token_end: int | None = None) -> list[dict[str, Any]]:
    """Token units covering [suffix_start, token_end) (semantic_units.py:360-421)."""
    encoded = tokenizer(text, add_special_tokens=False, return_offsets_mapping=True)
    ids = [int(v) for v in encoded["input_ids"]]
    if ids != [int(v) for v in expected_token_ids]:
        raise RuntimeError("semantic unit tokenizer identity drift")
    end = len(ids) if token_end is None else int(token_end)
    offsets = [(int(a), int(b)) for a, b in encoded["offset_mapping"]]
    if not 0 <= int(suffix_start) < end <= len(ids):
        raise ValueError("semantic unit suffix start out of range")
    text_units = semantic_char_units(text)
    if not text_units:
        raise RuntimeError("semantic unit construction produced no units")
    runs: list[dict[str, Any]] = []
    k, key = 0, None
    for tok in range(int(suffix_start), end):
        a, b = offsets[tok]
        mid = a if b <= a else (a + b - 1) / 2.0
        while k + 1 < len(text_units) and mid >= text_units[k]["end"]:
            k += 1
        src = text_units[k]
        here = (src["container_id"], src["start"], src["end"])
        if here == key:
            runs[-1]["end"] = tok + 1
        else:
            runs.append(_unit(tok, tok + 1, src["container_id"], src["container_kind"], src["boundary_kind"]))
            key = here
    units = _merge_short([piece for run in runs for piece in _chunked(run, run["start"], run["end"])])
    if (not units or units[0]["start"] != int(suffix_start) or units[-1]["end"] != end
            or any(x["end"] != y["start"] for x, y in zip(units, units[1:]))
            or any(u["end"] - u["start"] > MAX_UNIT_TOKENS for u in units)):
        raise RuntimeError("semantic unit token partition drift")
    return units


# ---------------------------------------------------------------- allocation
def score_semantic_units(*, units: list[dict[str, Any]], token_scores) -> list[dict[str, Any]]:
    """Each unit with its score: the mean of its top min(4, length) token scores."""
    out = []
    for index, u in enumerate(units):
        vals = [float(v) for v in token_scores[u["start"]:u["end"]]]
        if not vals or not all(math.isfinite(v) for v in vals):
            raise RuntimeError("invalid semantic unit token scores")
        top = sorted(vals, reverse=True)[:min(UNIT_TOP_K, len(vals))]
        out.append(dict(u, unit_index=index, token_count=u["end"] - u["start"], unit_score=sum(top) / len(top),
                        score_top_k=len(top)))
    return out


def best_forward_causal_window(*, start: int, end: int, width: int, token_scores) -> dict[str, Any]:
    """The `width`-token window of [start, end) with the largest summed forward
    utility u_i = max(exp(s_i - max s), exp(-1/16) * u_{i-1})."""
    width, span = int(width), int(end) - int(start)
    if not 0 < width <= span:
        raise ValueError("invalid semantic unit partial-window width")
    vals = [float(v) for v in token_scores[start:end]]
    top = max(vals)
    decay = math.exp(-1.0 / CAUSAL_DECAY_TOKENS)
    util, carry = [], 0.0
    for v in vals:
        carry = max(math.exp(v - top), decay * carry)
        util.append(carry)
    total = sum(util[:width])
    best, best_total = 0, total
    for s in range(1, span - width + 1):
        total += util[s + width - 1] - util[s - 1]
        if total > best_total:
            best, best_total = s, total
    return {"start": int(start) + best, "end": int(start) + best + width, "utility": best_total,
            "decay_tokens": CAUSAL_DECAY_TOKENS}


def select_semantic_unit_support(*, units: list[dict[str, Any]], token_scores,
                                 budget_tokens: int) -> tuple[list[int], dict[str, Any]]:
    """Exact-budget allocation over scored units (semantic_units.py:488-576)."""
    if not units:
        raise ValueError("semantic unit refresh requires units")
    lo, hi = units[0]["start"], units[-1]["end"]
    budget = min(max(1, int(budget_tokens)), hi - lo)
    scored = score_semantic_units(units=units, token_scores=token_scores)
    order = sorted(scored, key=lambda u: (-float(u["unit_score"]), u["start"]))
    support: list[int] = []
    picks = []
    for rank, u in enumerate(order):
        room = budget - len(support)
        if room <= 0:
            break
        if u["end"] - u["start"] <= room:
            window, kind, taken = None, "complete_unit", list(range(u["start"], u["end"]))
        else:
            window = best_forward_causal_window(start=u["start"], end=u["end"], width=room,
                                                token_scores=token_scores)
            kind, taken = "partial_forward_causal_window", list(range(window["start"], window["end"]))
        support += taken
        picks.append({"rank": rank, "unit_index": u["unit_index"], "unit_start": u["start"], "unit_end": u["end"],
                      "unit_score": float(u["unit_score"]), "selection_kind": kind, "selected_start": min(taken),
                      "selected_end": max(taken) + 1, "selected_tokens": len(taken), "partial_window": window})
    if len(support) != budget or len(set(support)) != budget:
        raise RuntimeError("semantic unit refresh support budget drift")
    # Metadata keys and rule texts are the reference's (part of the Selection contract).
    return sorted(support), {
        "revision": "SEMANTIC_UNIT_REFRESH_V1",
        "information_scope": "current query, edited prompt tokens, and deployable generic container/sentence "
                             "boundaries only",
        "kv_probe_token_calls": 0,
        "planning_expansion_token_calls": 0,
        "budget_tokens": budget,
        "unit_count": len(scored),
        "unit_score_rule": "mean of top min(4, unit_token_count) token scores",
        "long_unit_rule": "balanced fixed chunks with maximum 128 tokens",
        "short_unit_rule": "units shorter than 8 tokens merge with an adjacent unit in the same container when one "
                           "exists",
        "partial_unit_rule": "maximum-utility contiguous remaining-budget window under forward exponential causal "
                             "decay with 16-token scale",
        "units": scored,
        "selections": picks,
    }


# ------------------------------------------------------------------- scoring
def query_text_token_ids(tokenizer: Any, query_text: str) -> list[int]:
    ids = [int(v) for v in tokenizer(query_text, add_special_tokens=False)["input_ids"]]
    if not ids:
        raise ValueError("query text tokenization is empty")
    return ids


def _embedding_weight(model: Any) -> torch.Tensor:
    owner = getattr(model, "generator", model)
    return owner.get_input_embeddings().weight


@torch.no_grad()
def dense_query_relevance_scores(*, model: Any, edited_input_ids: torch.Tensor,
                                 query_token_ids: list[int]) -> tuple[list[float], dict[str, Any]]:
    """Per-token relevance of the edited prompt (scoring.py:11-72) on the GPU:
    one ``kvr_query_relevance`` call over the model's input embedding table
    (CUDA, bf16/fp16/fp32). ``model``: the model or an object whose
    ``generator`` is the model."""
    if not query_token_ids:
        raise ValueError("dense query scorer requires query tokens")
    table = _embedding_weight(model)
    if table.device.type != "cuda":
        raise ValueError("the B200 relevance scorer needs the embedding table on a CUDA device")
    codes = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16, torch.float32: _lib.DTYPE_F32}
    if table.dtype not in codes or table.dim() != 2 or not table.is_contiguous():
        raise ValueError("embedding table must be a contiguous 2-D bf16/fp16/fp32 tensor")
    device = table.device
    lib = _lib.load()
    prompt = edited_input_ids[0].to(device=device, dtype=torch.int64).contiguous()
    query = torch.tensor([int(v) for v in query_token_ids], dtype=torch.int64, device=device)
    vocab, hidden = table.shape
    need = lib.kvr_query_relevance_workspace_size(hidden, query.numel())
    workspace = torch.empty(need, dtype=torch.uint8, device=device)
    scores = torch.empty(prompt.numel(), dtype=torch.float32, device=device)
    with torch.cuda.device(device):
        _lib.check(lib.kvr_query_relevance(table.data_ptr(), vocab, hidden, codes[table.dtype], prompt.data_ptr(),
                                           prompt.numel(), query.data_ptr(), query.numel(), EXACT_TOKEN_BOOST,
                                           scores.data_ptr(), workspace.data_ptr(), need,
                                           _lib.stream_handle(device)), "query_relevance")
        bad = int(workspace[:4].view(torch.int32).item())
    if bad:
        raise IndexError("token id outside the embedding table")
    return [float(v) for v in scores.tolist()], {
        "query_token_ids": [int(v) for v in query_token_ids],
        "query_token_count": len(query_token_ids),
        "exact_token_boost": EXACT_TOKEN_BOOST,
        "embedding_dot_flops": 2 * int(prompt.numel()) * len(query_token_ids) * int(hidden),
        "embedding_dot_flops_scope": "prompt-token by query-token embedding dot products only; excludes lookup, "
                                     "normalization, max reduction, and exact-token boost",
    }


def sur_selector(model, tokenizer, text, query, ids, suffix_start, budget_percent):
    """The default allocator of ``select_support`` (api.py:83-96): units,
    B200 relevance scores, exact-budget allocation. Returns positions and
    metadata in the shape ``api._select_encoded`` expects."""
    length = int(ids.shape[1])
    suffix_tokens = length - suffix_start
    budget = min(suffix_tokens, math.ceil(suffix_tokens * budget_percent / 100.0))
    units = semantic_unit_token_ranges(tokenizer=tokenizer, text=text, expected_token_ids=ids[0].tolist(),
                                       suffix_start=suffix_start)
    scores, score_meta = dense_query_relevance_scores(model=model, edited_input_ids=ids,
                                                      query_token_ids=query_text_token_ids(tokenizer, query))
    positions, alloc_meta = select_semantic_unit_support(units=units, token_scores=scores, budget_tokens=budget)

    class _Picked:
        pass

    picked = _Picked()
    picked.positions = positions
    picked.metadata = {"selection": "sur", "scoring": score_meta, "allocator": alloc_meta}
    return picked
