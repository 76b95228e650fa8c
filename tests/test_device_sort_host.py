"""The per-target bucket sort of the target-ordered delivery kernel
(b2_sift_u64 / b2_sort_u64 in csrc/kernels/device_lib.cuh), compiled for the
host from the same source text and checked against std::sort on random keys
of every length from 0 to 300 (insertion sort up to 16, heapsort beyond)."""
from __future__ import annotations

import re
import subprocess

from conftest import ROOT

LIB = ROOT / "brian2-atlas_b200" / "csrc" / "kernels" / "device_lib.cuh"

MAIN = r"""
#include <algorithm>
#include <cstdio>
#include <random>
#include <vector>
typedef unsigned long long u64;
typedef unsigned int u32;
@BODY@
int main() {
  std::mt19937_64 rng(7);
  for (u32 n = 0; n <= 300; ++n) {
    for (int rep = 0; rep < 20; ++rep) {
      std::vector<u64> a(n);
      for (auto& x : a) x = rep % 2 ? rng() : rng() % 8;  // distinct-ish and heavily repeated keys
      std::vector<u64> want(a);
      std::sort(want.begin(), want.end());
      b2_sort_u64(a.data(), n);
      if (a != want) { std::printf("mismatch at n=%u\n", n); return 1; }
    }
  }
  std::printf("ok\n");
  return 0;
}
"""


def test_bucket_sort_matches_std_sort(tmp_path):
    text = LIB.read_text()
    start = text.index("__device__ __forceinline__ void b2_sift_u64")
    end = text.index("}\n}\n", text.index("__device__ inline void b2_sort_u64")) + 4
    body = re.sub(r"__device__ (__forceinline__|inline) ", "static inline ", text[start:end])
    src = tmp_path / "sort.cpp"
    src.write_text(MAIN.replace("@BODY@", body))
    exe = tmp_path / "sort"
    subprocess.run(["g++", "-O2", "-std=c++17", str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0 and out.stdout.strip() == "ok", out.stdout
