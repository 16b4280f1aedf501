"""Paged chunk cache of the Llama-family engine: allocation, deduplication by content, LRU
eviction to the host tier and page tables on CPU with a stand-in engine; on the GPU, an engine
reading its references through page tables equals the engine over a contiguous memory."""

from types import SimpleNamespace

import pytest
import torch

from pdattention_b200.inference.page_cache import PageAllocator, PagedChunkCache
from pdattention_b200.memory.services import create_device_cache


class _Encoder:
    """Stand-in engine: 'encodes' a chunk by writing its first token into its pool rows."""

    def __init__(self, layers=2, kv_dim=8, chunk_tokens=4):
        self.cfg = SimpleNamespace(num_hidden_layers=layers, chunk_tokens=chunk_tokens, kv_dim=kv_dim)
        self.kv_dim = kv_dim
        self.device = torch.device("cpu")
        self.encoded = []
        self.table = None

    def encode_into(self, mem, chunks, lengths, first, batch_chunks=256):
        self.encoded.append((first, chunks.shape[0]))
        mem.chunk_len[first: first + chunks.shape[0]] = lengths
        for i in range(chunks.shape[0]):
            mem.pool[:, (first + i) * mem.tc:(first + i + 1) * mem.tc] = float(chunks[i, 0])
            mem.gn_bf16[:, first + i] = float(chunks[i, 0])

    def set_page_table(self, table, counts):
        self.table = (table, counts)


def test_allocator_first_fit_and_merge():
    a = PageAllocator(10)
    assert (a.allocate(4), a.allocate(3), a.allocate(4)) == (0, 4, None)
    a.release(0, 4)
    a.release(4, 3)
    assert a.free == [[0, 10]] and a.allocate(10) == 0


def test_dedup_lru_eviction_and_host_restore():
    eng = _Encoder()
    cache = PagedChunkCache(eng, capacity_pages=6, host_capacity_pages=6)
    a = cache.add([1] * 8, uri="a")        # 2 pages
    b = cache.add([2] * 12, uri="b")       # 3 pages
    again = cache.add([1] * 8, uri="a2")   # same content: same pages, no encode
    assert again is a and a.refs == 2 and len(eng.encoded) == 2 and cache.stats["reused_entries"] == 1
    cache.release("a")
    cache.release(again)
    cache.release(b)
    c = cache.add([3] * 8, uri="c")        # needs 2 pages: evicts the least recently released (a)
    assert cache.stats["evicted_entries"] == 1 and "a" not in cache.by_uri and c.first == a.first
    assert float(cache.memory.pool[0, c.first * 4, 0]) == 3.0
    cache.release(c)
    restored = cache.add([1] * 8, uri="a")  # comes back from the host tier, not re-encoded
    assert cache.stats["restored_entries"] == 1 and len(eng.encoded) == 3
    assert float(cache.memory.pool[0, restored.first * 4, 0]) == 1.0
    assert [int(x) for x in cache.memory.chunk_len[restored.first: restored.first + 2]] == [4, 4]


def test_page_table_lists_each_rows_pages():
    eng = _Encoder()
    cache = PagedChunkCache(eng, capacity_pages=8)
    a, b, c = cache.add([1] * 5), cache.add([2] * 4), cache.add([3] * 9)
    table, counts = cache.page_table([[a, c], [b], []])
    assert counts.tolist() == [5, 1, 0]
    assert table[0, :5].tolist() == list(range(a.first, a.first + 2)) + list(range(c.first, c.first + 3))
    assert table[1, 0].item() == b.first and eng.table is not None


def test_full_pool_of_referenced_entries_raises():
    cache = PagedChunkCache(_Encoder(), capacity_pages=2)
    cache.add([1] * 8)
    with pytest.raises(RuntimeError, match="every entry is referenced"):
        cache.add([2] * 4)


def test_service_registry_builds_the_paged_cache():
    cache = create_device_cache(_Encoder(), {"type": "paged", "options": {"capacity_pages": 3}})
    assert isinstance(cache, PagedChunkCache) and cache.allocator.capacity == 3


@pytest.mark.gpu
def test_engine_over_page_tables_equals_contiguous_memory():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from pdattention_b200.inference.llama_engine import LlamaWeights, PRALlamaEngine
    from pdattention_b200.models.llama import PRALlamaReference, tiny_llama

    torch.manual_seed(0)
    cfg = tiny_llama(head_dim=64, hidden_size=128, num_attention_heads=4, num_key_value_heads=2, chunk_tokens=16,
                     top_k_chunks=3)
    model = PRALlamaReference(cfg).eval()
    model.reset_parameters(seed=0, std=0.08)
    weights = LlamaWeights.from_reference(model, "cuda")
    refs = [torch.randint(0, cfg.vocab_size, (n,)).tolist() for n in (40, 27, 64)]
    ids = torch.randint(0, cfg.vocab_size, (2, 12))
    plen = torch.tensor([12, 9])
    # contiguous memory: the three references' chunks back to back, rows 0 -> refs 0+1, row 1 -> ref 2
    base = PRALlamaEngine(weights, "cuda", decode_split_keys=64)
    chunks, lengths = [], []
    for r in refs:
        for i in range(0, len(r), 16):
            piece = r[i: i + 16]
            chunks.append(piece + [0] * (16 - len(piece)))
            lengths.append(len(piece))
    base.build_memory(torch.tensor(chunks), torch.tensor(lengths, dtype=torch.int32))
    base.set_namespace(torch.tensor([0, 5]), torch.tensor([5, 9]))
    want = base.prefill(ids, plen, 3).float()
    want_step = base.decode_step(want.argmax(-1)).float()
    # paged: the same references through the page cache (one duplicate added twice)
    paged = PRALlamaEngine(weights, "cuda", decode_split_keys=64)
    cache = PagedChunkCache(paged, capacity_pages=32)
    e = [cache.add(r) for r in refs]
    assert cache.add(refs[0]) is e[0] and cache.stats["encoded_pages"] == 9
    cache.page_table([[e[0], e[1]], [e[2]]])
    got = paged.prefill(ids, plen, 3).float()
    got_step = paged.decode_step(got.argmax(-1)).float()
    # same selections (below) and the same logits up to bf16 rounding: each reference encoded on its
    # own takes the <= 64-row decode GEMM (SwiGLU in its epilogue) where the back-to-back encode
    # of all nine chunks takes the large-batch GEMM and a separate SwiGLU pass
    assert torch.allclose(got, want, atol=3e-2, rtol=1e-2), (got - want).abs().max()
    assert torch.allclose(got_step, want_step, atol=3e-2, rtol=1e-2), (got_step - want_step).abs().max()
    for li in base.last_selection:
        assert torch.equal(paged.last_selection[li], base.last_selection[li])
