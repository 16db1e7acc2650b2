"""Background tokenizer: windows from a token stream built on a worker thread (CPU)."""
import pytest
import torch

from complexity_framework_b200.data import BackgroundTokenizer
from complexity_framework_b200.data.tokenization import ByteTokenizer


def test_windows_cover_the_stream_with_one_token_overlap():
    tok = ByteTokenizer()
    bg = BackgroundTokenizer(tok, max_length=8, buffer_size=4, eos_id=0)
    texts = [f"text number {i}" for i in range(20)]
    for t in texts:
        bg.submit(t)
    bg.close()
    stream = []
    for t in texts:
        stream += list(tok.encode(t)) + [0]
    wins = list(bg)
    assert all(w.shape == (9,) and w.dtype == torch.long for w in wins)
    for i, w in enumerate(wins):
        assert w.tolist() == stream[i * 8:i * 8 + 9]
    assert len(wins) == (len(stream) - 1) // 8
    assert bg.get_batch() is None


def test_errors_surface_to_consumer():
    class Bad:
        def encode(self, s):
            raise ValueError("boom")

    bg = BackgroundTokenizer(Bad(), max_length=4)
    bg.submit("x")
    with pytest.raises(RuntimeError):
        bg.get_batch(block=True, timeout=5)
