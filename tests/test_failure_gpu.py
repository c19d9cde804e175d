"""Device-side failure detection on one GPU: a bounded wait runs out and the host sees it.

The expert-parallel exchange waits for flags that peers publish. Here the wait is given a flag that
nothing sets and a 1 ms limit: the kernel must give up, record the timeout in the error flag and
return, so ``check_kernel_errors`` raises and the CUDA context stays usable. No GPU fault, trap or
hang is involved.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _flags():
    # one rank's flag area: [purpose][16 sources] int32, all zero (nothing ever published)
    return torch.zeros(256, dtype=torch.int32, device="cuda")


def test_peer_wait_times_out_and_reports():
    from marin_experiments_b200.ops._ext import KernelTimeoutError, check_kernel_errors, err_flag, ext

    flags = _flags()
    check_kernel_errors()  # start clean
    ext().ep_wait([flags.data_ptr()], 0, 0, 1, 1, err_flag(flags.device), 1_000_000)  # epoch 1 never arrives
    torch.cuda.synchronize()
    with pytest.raises(KernelTimeoutError, match="code 4"):
        check_kernel_errors()
    # the context is still usable and the flag was cleared
    x = torch.arange(10, device="cuda", dtype=torch.float32)
    assert float((x * 2).sum()) == 90.0
    check_kernel_errors()


def test_peer_wait_returns_when_flag_is_published():
    from marin_experiments_b200.ops._ext import check_kernel_errors, err_flag, ext

    flags = _flags()
    flags[1 * 16 + 0] = 3  # purpose 1, source 0 already at epoch 3
    ext().ep_wait([flags.data_ptr()], 0, 0, 1, 2, err_flag(flags.device), 1_000_000)
    torch.cuda.synchronize()
    check_kernel_errors()
