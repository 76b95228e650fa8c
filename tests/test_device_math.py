"""Device helpers checked element by element on the GPU (needs a GPU).

b2_binomial_thr (inversion decided by integer thresholds on the draw's bits,
the PoissonInput draw) against the loop it replaces, b2_binomial_inv, which
restates the reference's counter_binomial (executor.rs:224-268): identical
results for every counter of a large sample, at the configs' (n, p) and at a
reversed p > 0.5.  The thresholds are built here the way the plan compiler
builds them (bisection on the loop's own rounded subtractions).
"""
from __future__ import annotations

import ctypes
import math

import pytest

pytestmark = pytest.mark.gpu

KERNEL = r"""
extern "C" __global__ void compare_binomial(const u64* thr, double prob, double q, double qn,
                                            double bound, u64 n, int reverse, u64 count, u64* mismatches) {
  for (u64 i = blockIdx.x * (u64)blockDim.x + threadIdx.x; i < count; i += (u64)gridDim.x * blockDim.x) {
    const u64 tick = i >> 12, index = (i & 4095ull) * 7919ull;
    const double a = b2_binomial_inv(3ull, 5ull, tick, index, n, prob, q, qn, bound, reverse != 0);
    const double b = b2_binomial_thr<KSIZE>(3ull, 5ull, tick, index, n, thr, reverse != 0);
    if (__double_as_longlong(a) != __double_as_longlong(b)) atomicAdd(mismatches, 1ull);
  }
}
"""


def inversion_constants(n: int, p: float):
    reverse = p > 0.5
    prob = 1.0 - p if reverse else p
    q = 1.0 - prob
    qn = math.exp(n * math.log(q))
    bound = min(float(n), n * prob + 10.0 * math.sqrt(n * prob * q + 1.0))
    k = int(math.floor(bound)) + 1
    tab = [qn]
    for x in range(1, k):
        tab.append((float(n - x + 1) * prob * tab[-1]) / (float(x) * q))
    return reverse, prob, q, qn, bound, tab


def thresholds(tab):
    """Per x the largest m < 2^53 whose draw passes the loop's test at x,
    then the running maximum (the plan compiler's construction)."""
    out, run = [], 0
    for x in range(len(tab)):
        def passes(m):
            u = float(m) * 2.0 ** -53
            for j in range(x):
                u -= tab[j]
            return u <= tab[x]
        lo, hi = 0, 2 ** 53 - 1
        if passes(hi):
            lo = hi
        else:
            while hi - lo > 1:
                mid = (lo + hi) // 2
                if passes(mid):
                    lo = mid
                else:
                    hi = mid
        run = max(run, lo)
        out.append(run)
    return out


@pytest.mark.parametrize("n,p", [(100, 0.001), (800, 0.0025), (50, 0.3), (20, 0.7)])
def test_binomial_table_matches_inversion_loop(n, p):
    torch = pytest.importorskip("torch")
    from devkernel import Kernel
    dev = torch.device("cuda", 0)
    torch.cuda.init()
    reverse, prob, q, qn, bound, tab = inversion_constants(n, p)
    d_thr = torch.tensor(thresholds(tab), dtype=torch.int64, device=dev)
    mism = torch.zeros(1, dtype=torch.int64, device=dev)
    count = 1 << 24
    k = Kernel(KERNEL.replace("KSIZE", f"{len(tab)}u"), "compare_binomial")
    k.launch(148 * 8, 256,
             [d_thr.data_ptr(), prob, q, qn, bound, n, int(reverse), count, mism.data_ptr()],
             [ctypes.c_void_p, ctypes.c_double, ctypes.c_double, ctypes.c_double, ctypes.c_double,
              ctypes.c_uint64, ctypes.c_int, ctypes.c_uint64, ctypes.c_void_p],
             torch.cuda.current_stream(dev).cuda_stream)
    torch.cuda.synchronize(dev)
    assert int(mism.cpu()[0]) == 0

