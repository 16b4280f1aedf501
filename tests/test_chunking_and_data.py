import pytest
import torch

from pdattention_b200.chunking import ChunkingConfig, partition_reference, partition_source
from pdattention_b200.config import PRAConfig
from pdattention_b200.data import PRACollator, PRADataModule, PRATokenizer, WordIdTokenizer
from pdattention_b200.data.generators import generate_hierarchical_tokens, generate_kv_qa
from pdattention_b200.data.schemas import QuestionSample, ReferenceSample

TEXT = "Alpha beta gamma.<PRA_CHUNK>Delta epsilon.<PRA_CHUNK>Zeta eta theta iota kappa lambda mu." * 3


def _chunks_equal(a, b):
    assert [(c.chunk_id, c.token_ids, c.token_start, c.token_end, c.char_start, c.char_end) for c in a] == \
           [(c.chunk_id, c.token_ids, c.token_start, c.token_end, c.char_start, c.char_end) for c in b]
    assert [c.metadata for c in a] == [c.metadata for c in b]


@pytest.mark.parametrize("policy", [
    {"mode": "none"}, {"mode": "fixed", "chunk_tokens": 16}, {"mode": "fixed", "chunk_tokens": 16, "overlap_tokens": 4},
    {"mode": "fixed", "chunk_tokens": 20, "overlap_fraction": 0.25}, {"mode": "markers"},
])
@pytest.mark.parametrize("cap,overflow", [(None, "truncate"), (3, "truncate"), (3, "merge_tail")])
def test_partition_source_matches_reference(ref, policy, cap, overflow):
    tok = PRATokenizer([TEXT])
    ids = tok.encode(TEXT)
    mine = partition_source("mem://d", ids, tok, ChunkingConfig(**policy), {"k": 1}, text=TEXT, max_chunks=cap,
                            overflow_policy=overflow, max_chunk_tokens=40)
    theirs = ref.chunking.partition_source("mem://d", ids, tok, ref.chunking.ChunkingConfig(**policy), {"k": 1},
                                           text=TEXT, max_chunks=cap, overflow_policy=overflow, max_chunk_tokens=40)
    _chunks_equal(mine, theirs)


def test_partition_reference_uses_config_cap(ref):
    tok = PRATokenizer([TEXT])
    kw = dict(chunking_mode="fixed", fixed_chunk_tokens=12, max_gists_per_reference=5)
    _chunks_equal(partition_reference("u", TEXT, tok, PRAConfig(**kw)),
                  ref.chunking.partition_reference("u", TEXT, tok, ref.config.PRAConfig(**kw)))


def test_chunk_ids_are_stable_and_exact():
    tok = PRATokenizer([TEXT])
    ids = tok.encode(TEXT)
    chunks = partition_source("u", ids, tok, ChunkingConfig(mode="fixed", chunk_tokens=10))
    assert [t for c in chunks for t in c.token_ids] == ids
    assert chunks[10].chunk_id == "u#chunk=10"


def test_tokenizer_and_collator_match_reference(ref):
    texts = ["Which animal hunts mice? <REF_1> <REF_2>", "cat", "Facts <REF_7>"]
    mine, theirs = PRATokenizer(texts), ref.tokenizer.PRATokenizer(texts)
    assert mine.stoi == theirs.stoi
    assert mine.encode(texts[0] + "é<REF_9>") == theirs.encode(texts[0] + "é<REF_9>")
    samples = [QuestionSample("q1", "Which animal hunts mice? <REF_1> <REF_2>", "cat",
                              [ReferenceSample(1, "mem://a", "s", metadata={"text": "x"})], [1]),
               QuestionSample("q2", "Long " * 30, "dog", [], [])]
    a = PRACollator(mine, max_seq_len=40)(samples)
    b = ref.collators.PRACollator(theirs, max_seq_len=40)(samples)
    for key in ("input_ids", "labels", "attention_mask"):
        assert torch.equal(a[key], b[key])
    assert a["metadata"][1]["full_input_ids"] == b["metadata"][1]["full_input_ids"]
    assert a["metadata"][1]["full_labels"] == b["metadata"][1]["full_labels"]


def test_word_id_tokenizer_roundtrip():
    tok = WordIdTokenizer(1000)
    ids = tok.encode("t5 t999 <REF_3> t17")
    assert ids[:2] == [5, 999] and ids[2] >= 1000 and tok.decode(ids) == "t5 t999 <REF_3> t17"


def test_kv_qa_stage_shape(tmp_path):
    generate_kv_qa(tmp_path / "synthetic_kv_qa", n=6, seed=3)
    dm = PRADataModule("synthetic_kv_qa", str(tmp_path), batch_size=2, max_seq_len=128).load()
    for sample in dm.dataset:
        assert 2 <= len(sample.references) <= 4
        for ref_sample in sample.references:
            text = ref_sample.metadata["text"]
            assert text.count(":") >= 8 and 256 <= len(text)
        assert sample.target_reference_ids


def test_hierarchical_token_stage_has_sixteen_refs(tmp_path):
    generate_hierarchical_tokens(tmp_path / "synthetic_hierarchical_tokens", examples=2, doc_tokens=32,
                                 prompt_tokens=40, vocab=500)
    dm = PRADataModule("synthetic_hierarchical_tokens", str(tmp_path), batch_size=2, max_seq_len=64,
                       tokenizer=WordIdTokenizer(500)).load()
    sample = dm.dataset[0]
    assert len(sample.references) == 2
    documents = sample.references[0].metadata["documents"]
    own = [u for u in documents if u.startswith("tree://e0/")]
    assert len(own) == 16
