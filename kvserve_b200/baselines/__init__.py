"""Baseline arms used by the benchmarks (the reference's own build and the
uncompressed NCCL hand-off)."""
