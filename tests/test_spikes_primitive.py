"""b2g_spikes_from_bitmap: device bitmap -> ascending spike ids (needs a GPU).

Checked against numpy's nonzero on the same seeded bitmaps: empty, one bit,
word and tile boundaries, ragged tails whose bits past nbits are set (they
must be ignored), dense and sparse fills, and a 2^24-neuron population.
Torch allocates the device buffers (plumbing); the work is the library's.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SIZES = [0, 1, 31, 32, 33, 1000, 32 * 1024 * 4 + 5, 1_000_000, (1 << 24) + 3]


def expected_ids(words: np.ndarray, nbits: int) -> np.ndarray:
    bits = np.unpackbits(words.view(np.uint8), bitorder="little")[:nbits]
    return np.flatnonzero(bits).astype(np.uint32)


def run(pkg, torch, words: np.ndarray, nbits: int):
    dev = torch.device("cuda", 0)
    d_words = torch.from_numpy(words.view(np.int32)).to(dev) if words.size else torch.zeros(1, dtype=torch.int32,
                                                                                            device=dev)
    d_ids = torch.full((max(nbits, 1),), -1, dtype=torch.int32, device=dev)
    d_count = torch.full((1,), -1, dtype=torch.int32, device=dev)
    nscratch = pkg.spikes_scratch_bytes(nbits)
    d_scratch = torch.empty(nscratch, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    pkg.spikes_from_bitmap(d_words.data_ptr(), nbits, d_ids.data_ptr(), d_count.data_ptr(), d_scratch.data_ptr(),
                           nscratch, stream.cuda_stream)
    torch.cuda.synchronize(dev)
    n = int(d_count.cpu()[0])
    return n, d_ids.cpu().numpy().view(np.uint32)[:n]


@pytest.mark.parametrize("nbits", SIZES)
@pytest.mark.parametrize("density", [0.001, 0.3, 1.0])
def test_matches_numpy(pkg, nbits, density):
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(nbits * 7 + int(density * 1000))
    nwords = (nbits + 31) // 32
    bits = (rng.random(nwords * 32) < density).astype(np.uint8)  # includes bits past nbits
    words = np.packbits(bits, bitorder="little").view(np.uint32).copy()
    n, ids = run(pkg, torch, words, nbits)
    want = expected_ids(words, nbits)
    assert n == len(want)
    assert np.array_equal(ids, want)


def test_undersized_scratch_is_rejected(pkg):
    torch = pytest.importorskip("torch")
    dev = torch.device("cuda", 0)
    buf = torch.zeros(1 << 20, dtype=torch.int32, device=dev)
    with pytest.raises(pkg.B2GpuError, match="scratch"):
        pkg.spikes_from_bitmap(buf.data_ptr(), 1 << 24, buf.data_ptr(), buf.data_ptr(), buf.data_ptr(), 8, 0)
