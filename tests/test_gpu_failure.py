"""A device-side wait that runs out ends as a status word and an error row (GPU).

Every probe kernel waits on mbarriers with a bounded wait; when one runs out
the kernel writes TCB_ERR_TIMEOUT into its status word and returns.  These
tests make such a wait run out on purpose, on an mbarrier armed for bytes no
copy delivers (tcb_selftest_bounded_wait, with a 1 ms limit), and check:

* the status word reads TCB_ERR_TIMEOUT, the launch returns within a fraction
  of a second, and the context stays usable (a copy afterwards is exact);
* the tensor driver turns a nonzero status word into a failure, and the suite
  runner turns that child's failure into an `error` row of the table.

No trap, no fault, no hang: the kernel returns by itself.
"""

from pathlib import Path
import time
from types import SimpleNamespace

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_runs_out_and_reports(cuda, native):
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    torch.cuda.synchronize()
    start = time.perf_counter()
    native.selftest_bounded_wait(1_000_000, status)
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - start
    assert int(status.item()) == native.ERR_TIMEOUT
    assert "timed out" in native.strerror(int(status.item()))
    assert elapsed < 0.5, elapsed
    # The context is still usable.
    src = torch.randint(0, 256, (1 << 20,), dtype=torch.uint8, device=cuda)
    dst = torch.zeros_like(src)
    native.copy(src, dst, src.numel(), native.COPY_BULK)
    torch.cuda.synchronize()
    assert torch.equal(src, dst)


def test_status_word_keeps_the_first_error(cuda, native):
    status = torch.full((1,), native.ERR_DEVICE, dtype=torch.int32, device=cuda)
    native.selftest_bounded_wait(1_000_000, status)
    torch.cuda.synchronize()
    assert int(status.item()) == native.ERR_DEVICE


def test_timeout_becomes_an_error_row(cuda, native, monkeypatch, tmp_path):
    from triton_chip_benchmarks_b200 import bench_suite, bench_tensor, suite_report

    real_launch = bench_tensor.launch

    def launch_then_time_out(key, config, a, b, c, extras, blocks, blocks_per_sm, iterations,
                             status=None):
        real_launch(key, config, a, b, c, extras, blocks, blocks_per_sm, iterations, status)
        native.selftest_bounded_wait(1_000_000, status)

    monkeypatch.setattr(bench_tensor, "launch", launch_then_time_out)
    output = tmp_path / "tensor_bf16.json"
    with pytest.raises(RuntimeError, match="timed out"):
        bench_tensor.main(["--mode", "peak", "--dtype", "bf16", "--quick", "--device", "0",
                           "--output", str(output)])
    assert not output.exists()
    # The child exits non-zero without a document: the suite records an error row.
    metric = next(m for m in suite_report.METRICS if m.key == "tensor_bf16")
    row, document = bench_suite.conclude(metric, SimpleNamespace(quick=True), Path(output), 1)
    assert row["status"] == "error" and document is None
