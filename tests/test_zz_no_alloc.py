"""b2g_spikes_from_bitmap_noalloc against b2g_spikes_from_bitmap (needs a GPU).

The no-alloc entry point keeps its scratch in a fixed device array of the
library; it must give exactly the result of the entry point that takes a
caller scratch buffer, on two calls in a row on different bitmaps (the second
call reuses the array the first one left behind), and reject bitmaps above its
size limit.  This file is collected last, so it also runs after every other
test in the same process.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _bitmap(torch, dev, nbits, density, seed):
    rng = np.random.default_rng(seed)
    nwords = max((nbits + 31) // 32, 1)
    bits = (rng.random(nwords * 32) < density).astype(np.uint8)
    words = np.packbits(bits, bitorder="little").view(np.int32).copy()
    return torch.from_numpy(words).to(dev)


def _with_scratch(pkg, torch, dev, d_words, nbits):
    ids = torch.full((max(nbits, 1),), -1, dtype=torch.int32, device=dev)
    count = torch.full((1,), -1, dtype=torch.int32, device=dev)
    n = pkg.spikes_scratch_bytes(nbits)
    scratch = torch.empty(n, dtype=torch.uint8, device=dev)
    pkg.spikes_from_bitmap(d_words.data_ptr(), nbits, ids.data_ptr(), count.data_ptr(), scratch.data_ptr(), n,
                           torch.cuda.current_stream(dev).cuda_stream)
    return ids, count


def _no_alloc(pkg, torch, dev, d_words, nbits):
    ids = torch.full((max(nbits, 1),), -1, dtype=torch.int32, device=dev)
    count = torch.full((1,), -1, dtype=torch.int32, device=dev)
    pkg.spikes_from_bitmap_noalloc(d_words.data_ptr(), nbits, ids.data_ptr(), count.data_ptr(),
                                   torch.cuda.current_stream(dev).cuda_stream)
    return ids, count


@pytest.mark.parametrize("nbits", [0, 33, 1_000_000, 1 << 27])
def test_no_alloc_matches_scratch_entry_point_twice(pkg, nbits):
    torch = pytest.importorskip("torch")
    dev = torch.device("cuda", 0)
    for call, density in enumerate([0.01, 0.5]):  # two calls in a row, different data
        d_words = _bitmap(torch, dev, nbits, density, seed=nbits + call)
        ids_a, count_a = _with_scratch(pkg, torch, dev, d_words, nbits)
        ids_b, count_b = _no_alloc(pkg, torch, dev, d_words, nbits)
        torch.cuda.synchronize(dev)
        n = int(count_a.cpu()[0])
        assert int(count_b.cpu()[0]) == n
        assert torch.equal(ids_a[:n], ids_b[:n])


def test_no_alloc_rejects_bitmaps_above_its_limit(pkg):
    torch = pytest.importorskip("torch")
    dev = torch.device("cuda", 0)
    buf = torch.zeros(16, dtype=torch.int32, device=dev)
    with pytest.raises(pkg.B2GpuError, match="no-alloc limit"):
        pkg.spikes_from_bitmap_noalloc(buf.data_ptr(), pkg.SPIKES_NOALLOC_MAX_BITS + 1, buf.data_ptr(),
                                       buf.data_ptr())
