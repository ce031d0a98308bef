"""One-process-per-GPU pipeline (torchrun): placeholder until the IPC stage runner lands."""


def run_bench_multi(*a, **k):
    raise NotImplementedError("multi-GPU pipeline bench is not built yet")
