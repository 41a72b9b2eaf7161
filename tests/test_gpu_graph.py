"""CUDA-graph replay of repeated refresh requests (``graph_replay``): a
request that repeats an earlier one's geometry and buffers is captured once
and replayed, with the bytes of direct launches, with each request's own ids
and positions, and with its kernels counted."""

import pytest
import torch

from conftest import load_golden
from helpers import bits_equal, fixture_model, layers_cpu, to_cache

pytestmark = pytest.mark.gpu
DEV = "cuda"
CASES = ["case_qwen3_bf16_d128.pt", "case_llama_bf16_d64.pt"]


@pytest.fixture(autouse=True)
def _fresh_graph_cache():
    """Each test starts with no cached graph, so that a graph captured by an
    earlier test at the same addresses cannot shift the replay counts."""
    from budgeted_kv_cache_repair_b200 import engine

    engine.release_graphs()
    yield
    engine.release_graphs()


@pytest.fixture(params=["cublas", "sm100", "fused"])
def projections(request, monkeypatch):
    from budgeted_kv_cache_repair_b200 import _lib, engine

    monkeypatch.setattr(engine, "PROJECTIONS", {"cublas": _lib.PROJ_CUBLAS, "sm100": _lib.PROJ_SM100,
                                                "fused": _lib.PROJ_FUSED}[request.param])
    return request.param


def _setup(name):
    from budgeted_kv_cache_repair_b200 import OperatorShim

    record = load_golden(name)
    model = fixture_model(record, DEV)
    return record, OperatorShim(model), to_cache(record["shifted_layers"], DEV)


def _direct(monkeypatch, shim, base, ids, intervals):
    from budgeted_kv_cache_repair_b200 import engine, packed_interval_repair

    monkeypatch.setattr(engine, "GRAPH_REPLAY", False)
    out, _ = packed_interval_repair(shim, base, ids, intervals)
    got = layers_cpu(out)
    monkeypatch.setattr(engine, "GRAPH_REPLAY", True)
    return got


def _same(a, b):
    return all(bits_equal(x, y) for pa, pb in zip(a, b) for x, y in zip(pa, pb))


def _counters():
    from budgeted_kv_cache_repair_b200 import _lib

    lib = _lib.load()
    torch.cuda.synchronize()
    return lib.kvr_graph_replays(), lib.kvr_kernel_launches()


@pytest.mark.parametrize("name", CASES)
def test_replay_gives_the_bytes_of_direct_launches(name, projections, monkeypatch):
    from budgeted_kv_cache_repair_b200 import packed_interval_repair

    record, shim, base = _setup(name)
    ids = record["new_ids"].to(DEV)
    expect = _direct(monkeypatch, shim, base, ids, record["intervals"])
    replays0, launches0 = _counters()
    per_call = []
    for _ in range(5):
        before = _counters()[1]
        out, _ = packed_interval_repair(shim, base, ids, record["intervals"])
        assert _same(layers_cpu(out), expect)
        del out  # the next call gets the same output buffers back: same launch key
        per_call.append(_counters()[1] - before)
    replays, _ = _counters()
    # Call 1 runs directly (first sight of the key), call 2 captures and
    # launches the graph, calls 3-5 replay it.
    assert replays - replays0 == 4
    assert len(set(per_call)) == 1 and per_call[0] > 0  # a replay counts the kernels it runs


@pytest.mark.parametrize("name", CASES)
def test_replay_reads_each_requests_ids_and_positions(name, monkeypatch):
    """Same geometry (rows, last position), other positions and ids: the
    staged values reach the replayed kernels."""
    from budgeted_kv_cache_repair_b200 import packed_interval_repair

    record, shim, base = _setup(name)
    ids_a = record["new_ids"].to(DEV)
    intervals_a = [tuple(i) for i in record["intervals"]]
    # Move an inner interval one row earlier (still sorted, disjoint and
    # non-adjacent; the last row stays) and change the token ids it covers.
    i = next(j for j in range(1, len(intervals_a) - 1) if intervals_a[j][0] - 1 > intervals_a[j - 1][1])
    s0, e0 = intervals_a[i]
    intervals_b = intervals_a[:i] + [(s0 - 1, e0 - 1)] + intervals_a[i + 1:]
    ids_b = ids_a.clone()
    ids_b[0, s0 - 1:e0 - 1] = (ids_b[0, s0 - 1:e0 - 1] + 7) % int(shim.generator.config.vocab_size)
    expect_a = _direct(monkeypatch, shim, base, ids_a, intervals_a)
    expect_b = _direct(monkeypatch, shim, base, ids_b, intervals_b)
    assert not _same(expect_a, expect_b)
    replays0, _ = _counters()
    for ids, intervals, expect in [(ids_a, intervals_a, expect_a), (ids_a, intervals_a, expect_a),
                                   (ids_b, intervals_b, expect_b), (ids_a, intervals_a, expect_a),
                                   (ids_b, intervals_b, expect_b)]:
        out, _ = packed_interval_repair(shim, base, ids, intervals)
        assert _same(layers_cpu(out), expect)
        del out
    assert _counters()[0] - replays0 == 4


def test_held_outputs_are_never_captured(monkeypatch):
    """Outputs the caller keeps are new buffers each call: every call runs
    directly and no graph is made."""
    from budgeted_kv_cache_repair_b200 import packed_interval_repair

    record, shim, base = _setup(CASES[0])
    ids = record["new_ids"].to(DEV)
    expect = _direct(monkeypatch, shim, base, ids, record["intervals"])
    replays0, _ = _counters()
    kept = [packed_interval_repair(shim, base, ids, record["intervals"])[0] for _ in range(3)]
    assert _counters()[0] == replays0
    for out in kept:
        assert _same(layers_cpu(out), expect)


def test_replay_leaves_the_base_cache_untouched(monkeypatch):
    from budgeted_kv_cache_repair_b200 import packed_interval_repair

    record, shim, base = _setup(CASES[0])
    snapshot = layers_cpu(base)
    ids = record["new_ids"].to(DEV)
    for _ in range(4):
        out, _ = packed_interval_repair(shim, base, ids, record["intervals"])
        del out
    assert _same(layers_cpu(base), snapshot)


def test_graphs_of_an_exited_thread_are_released(monkeypatch):
    """A worker thread captures and replays, then exits (its graphs are
    destroyed with it); the main thread's next calls are unaffected."""
    import threading

    from budgeted_kv_cache_repair_b200 import packed_interval_repair

    record, shim, base = _setup(CASES[0])
    ids = record["new_ids"].to(DEV)
    expect = _direct(monkeypatch, shim, base, ids, record["intervals"])
    results = []

    def worker():
        torch.cuda.set_device(0)
        for _ in range(3):
            out, _ = packed_interval_repair(shim, base, ids, record["intervals"])
            results.append(layers_cpu(out))
            del out

    replays0, _ = _counters()
    thread = threading.Thread(target=worker)
    thread.start()
    thread.join()
    assert len(results) == 3 and all(_same(r, expect) for r in results)
    assert _counters()[0] - replays0 == 2
    for _ in range(3):
        out, _ = packed_interval_repair(shim, base, ids, record["intervals"])
        assert _same(layers_cpu(out), expect)
        del out


def test_release_starts_over(monkeypatch):
    from budgeted_kv_cache_repair_b200 import engine, packed_interval_repair

    record, shim, base = _setup(CASES[0])
    ids = record["new_ids"].to(DEV)
    expect = _direct(monkeypatch, shim, base, ids, record["intervals"])

    def calls(n):
        start = _counters()[0]
        for _ in range(n):
            out, _ = packed_interval_repair(shim, base, ids, record["intervals"])
            assert _same(layers_cpu(out), expect)
            del out
        return _counters()[0] - start

    assert calls(3) == 2  # direct, capture + launch, replay
    engine.release_graphs()
    assert calls(1) == 0  # the key is new again: direct
    assert calls(1) == 1  # captured again


def test_threads_on_one_stream_keep_their_own_requests(monkeypatch):
    """Two threads issue requests of one geometry with different ids and
    positions on the same stream, interleaved: each gets its own result (the
    staged inputs are per thread)."""
    import threading

    from budgeted_kv_cache_repair_b200 import packed_interval_repair

    record, shim, base = _setup(CASES[0])
    ids_a = record["new_ids"].to(DEV)
    intervals_a = [tuple(i) for i in record["intervals"]]
    i = next(j for j in range(1, len(intervals_a) - 1) if intervals_a[j][0] - 1 > intervals_a[j - 1][1])
    s0, e0 = intervals_a[i]
    intervals_b = intervals_a[:i] + [(s0 - 1, e0 - 1)] + intervals_a[i + 1:]
    ids_b = ids_a.clone()
    ids_b[0, s0 - 1:e0 - 1] = (ids_b[0, s0 - 1:e0 - 1] + 11) % int(shim.generator.config.vocab_size)
    expect = {"a": _direct(monkeypatch, shim, base, ids_a, intervals_a),
              "b": _direct(monkeypatch, shim, base, ids_b, intervals_b)}
    request = {"a": (ids_a, intervals_a), "b": (ids_b, intervals_b)}
    barrier = threading.Barrier(2)
    failures = []

    def worker(name):
        torch.cuda.set_device(0)
        ids, intervals = request[name]
        barrier.wait()
        for _ in range(4):
            out, _ = packed_interval_repair(shim, base, ids, intervals)
            if not _same(layers_cpu(out), expect[name]):
                failures.append(name)
            del out

    threads = [threading.Thread(target=worker, args=(n,)) for n in ("a", "b")]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not failures, failures


def _word_tokenizer(words):
    from tokenizers import Tokenizer
    from tokenizers.models import WordLevel
    from tokenizers.pre_tokenizers import WhitespaceSplit
    from transformers import PreTrainedTokenizerFast

    backend = Tokenizer(WordLevel({w: i for i, w in enumerate(words)}, unk_token="[UNK]"))
    backend.pre_tokenizer = WhitespaceSplit()
    return PreTrainedTokenizerFast(tokenizer_object=backend, unk_token="[UNK]")


def test_in_place_refresh_of_repair_after_deletion_replays(monkeypatch):
    """repair_after_deletion refreshes the shifted cache it owns in place (no
    copy source): repeated calls replay that graph with the direct bytes."""
    from budgeted_kv_cache_repair_b200 import engine, repair_after_deletion
    from helpers import to_cache

    record = load_golden("api_llama_bfloat16.pt")
    tokenizer = _word_tokenizer(record["words"])
    model = fixture_model(record, DEV)
    old = to_cache(record["old_layers"], DEV)

    def call():
        result = repair_after_deletion(model, tokenizer, old, record["original_text"],
                                       delete_span=tuple(record["delete_span"]), query=record["query"],
                                       budget_percent=record["budget_percent"])
        return list(result.selection.positions), layers_cpu(result.cache)

    monkeypatch.setattr(engine, "GRAPH_REPLAY", False)
    positions, expect = call()
    monkeypatch.setattr(engine, "GRAPH_REPLAY", True)
    replays0, _ = _counters()
    for _ in range(4):
        got_positions, got = call()
        assert got_positions == positions and _same(got, expect)
    assert _counters()[0] - replays0 >= 2


@pytest.mark.parametrize("name", CASES)
def test_weights_changed_in_place_between_replays(name, monkeypatch):
    """Weights modified in place after a request's graph was captured are
    used by the next call: q/k/v (whose fused copy the engine owns and
    rebuilds when their version counters move) and o/MLP weights (read
    through their own storage). The result equals a direct run with the new
    weights and differs from the old one."""
    from budgeted_kv_cache_repair_b200 import packed_interval_repair

    record, shim, base = _setup(name)
    ids = record["new_ids"].to(DEV)
    for _ in range(3):  # direct, captured, replayed
        out, _ = packed_interval_repair(shim, base, ids, record["intervals"])
        before = layers_cpu(out)
        del out
    first, last = shim.generator.model.layers[0], shim.generator.model.layers[-1]
    with torch.no_grad():  # o and down of layer 0 reach every later layer's K/V
        last.self_attn.k_proj.weight.mul_(1.5)
        first.self_attn.o_proj.weight.mul_(0.5)
        first.mlp.down_proj.weight.mul_(2.0)
    out, _ = packed_interval_repair(shim, base, ids, record["intervals"])
    after = layers_cpu(out)
    del out
    expect = _direct(monkeypatch, shim, base, ids, record["intervals"])
    assert _same(after, expect)
    assert not _same(after, before)
