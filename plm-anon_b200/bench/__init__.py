"""Command-line tools of the B200 round engine: ``bench.generate`` (the reference's generation CLI) and
``bench.kernels`` (single-kernel microbenchmarks)."""
