// b2gpu-runner: drop-in replacement for the reference `b2-runner` binary.
// The Brian2/Atlas frontend selects it with B2_RUNNER=/path/to/b2gpu-runner
// (brian2-rust/python/brian2_rust/device.py:1316-1365 resolves B2_RUNNER and
// invokes `runner MODEL.json OUTDIR` as a subprocess).
#include "../../include/b2gpu.h"

int main(int argc, char** argv) { return b2g_run_cli(argc, argv); }
