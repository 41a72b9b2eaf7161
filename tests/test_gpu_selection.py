"""Query relevance on the B200 (``kvr_query_relevance``) and the full
``select_support`` / ``repair_after_deletion`` path with the engine's own SUR
allocator, against the reference's choices recorded in the api fixtures."""

import pytest
import torch
import torch.nn.functional as F

from conftest import load_golden
from helpers import fixture_model, layers_cpu, to_cache

pytestmark = pytest.mark.gpu
DEV = "cuda"


class _Model:
    def __init__(self, table):
        self.table = torch.nn.Embedding.from_pretrained(table, freeze=True)

    def get_input_embeddings(self):
        return self.table


def _torch_scores(table, prompt, query, boost=0.25):
    """scoring.py:11-72 restated with torch ops in fp32 (the test's reference)."""
    qv = F.normalize(table[query].float(), dim=-1)
    pv = F.normalize(table[prompt].float(), dim=-1)
    sim = (pv.double() @ qv.double().T).max(dim=1).values
    exact = torch.tensor([0.25 if int(t) in set(query.tolist()) else 0.0 for t in prompt.tolist()],
                         dtype=torch.float64, device=table.device)
    return (sim + exact).float()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("hidden, nq", [(64, 1), (4096, 3), (4096, 19), (520, 9), (8192, 5), (12288, 9)])
def test_relevance_kernel_matches_torch(dtype, hidden, nq):
    from budgeted_kv_cache_repair_b200.selection import dense_query_relevance_scores

    gen = torch.Generator(device=DEV).manual_seed(hidden + nq)
    table = torch.randn(997, hidden, device=DEV, generator=gen).to(dtype)
    table[5].zero_()  # a zero row: cosine 0 through the 1e-12 clamp
    prompt = torch.randint(0, 997, (1, 3001), device=DEV, generator=gen)
    prompt[0, :4] = 5
    query = torch.randint(0, 997, (nq,), device=DEV, generator=gen)
    prompt[0, 7] = query[0]
    got, meta = dense_query_relevance_scores(model=_Model(table), edited_input_ids=prompt,
                                             query_token_ids=query.tolist())
    want = _torch_scores(table, prompt[0], query)
    assert torch.allclose(torch.tensor(got, device=DEV), want, atol=2e-6, rtol=0), \
        (torch.tensor(got, device=DEV) - want).abs().max().item()
    assert meta["embedding_dot_flops"] == 2 * 3001 * nq * hidden


def test_reference_scoring_cases_on_the_gpu():
    """The reference's test_scoring.py cases (hidden padded from 2 to 8 with zeros)."""
    from budgeted_kv_cache_repair_b200.selection import dense_query_relevance_scores

    vectors = torch.zeros(4, 8, device=DEV)
    vectors[:, :2] = torch.tensor([[1.0, 0.0], [1.0, 0.0], [-1.0, 0.0], [0.0, 1.0]])
    model = _Model(vectors)
    scores, meta = dense_query_relevance_scores(model=model, edited_input_ids=torch.tensor([[0, 1, 2, 3]], device=DEV),
                                                query_token_ids=[1])
    assert scores == pytest.approx([1.0, 1.25, -1.0, 0.0])
    assert meta["exact_token_boost"] == 0.25
    prompt = torch.tensor([[2] * 1024 + [3]], device=DEV)
    scores, _ = dense_query_relevance_scores(model=model, edited_input_ids=prompt, query_token_ids=[1, 3])
    assert scores == pytest.approx([0.0] * 1024 + [1.25])
    with pytest.raises(ValueError, match="requires query tokens"):
        dense_query_relevance_scores(model=model, edited_input_ids=prompt, query_token_ids=[])
    with pytest.raises(IndexError):
        dense_query_relevance_scores(model=model, edited_input_ids=torch.tensor([[0, 9]], device=DEV),
                                     query_token_ids=[1])


def _word_tokenizer(words):
    from tokenizers import Tokenizer
    from tokenizers.models import WordLevel
    from tokenizers.pre_tokenizers import WhitespaceSplit
    from transformers import PreTrainedTokenizerFast

    backend = Tokenizer(WordLevel({w: i for i, w in enumerate(words)}, unk_token="[UNK]"))
    backend.pre_tokenizer = WhitespaceSplit()
    return PreTrainedTokenizerFast(tokenizer_object=backend, unk_token="[UNK]")


@pytest.mark.parametrize("name", ["api_llama_bfloat16.pt", "api_qwen3_bfloat16.pt"])
def test_repair_after_deletion_with_engine_selection_matches_reference(name):
    """No selector: the engine's SUR allocator picks the reference's positions."""
    from budgeted_kv_cache_repair_b200 import repair_after_deletion, select_support

    record = load_golden(name)
    tokenizer = _word_tokenizer(record["words"])
    model = fixture_model(record, DEV)
    old = to_cache(record["old_layers"], DEV)
    result = repair_after_deletion(model, tokenizer, old, record["original_text"],
                                   delete_span=tuple(record["delete_span"]), query=record["query"],
                                   budget_percent=record["budget_percent"])
    assert list(result.selection.positions) == record["positions"]
    assert result.selection.metadata["selection"] == "sur"
    assert result.selection.metadata["allocator"]["revision"] == "SEMANTIC_UNIT_REFRESH_V1"
    again = select_support(model, tokenizer, record["edited_text"], record["query"],
                           suffix_start=record["suffix_start"], budget_percent=record["budget_percent"])
    assert list(again.positions) == record["positions"]
    assert len(layers_cpu(result.cache)) == len(record["old_layers"])
