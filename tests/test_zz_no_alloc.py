"""The allocation-free normalisation entry point, called through the C ABI.

Some callers cannot allocate device memory when they normalise (another
component owns every allocation through its own pool, or an allocation could
block or fail in the middle of a step), so ``gns_frobenius_normalize_noalloc``
keeps its scratch in a fixed array inside the library instead of a caller
workspace. This test checks that it returns exactly what the workspace-taking
entry point ``gns_frobenius_normalize`` returns, on two calls in a row with
different inputs (the second call must not see the first call's leftovers in
the shared scratch), that repeated calls leave the device's free memory
unchanged (nothing is allocated), that a batch close to its 8192-matrix limit
is served, and that a larger batch is refused with a message. It is collected
last so that a failure here does not hide the other tests.
"""

from __future__ import annotations

import pytest
import torch

from gram_newton_schulz_ampere_b200 import _native

pytestmark = pytest.mark.gpu

F16 = 0
CODES = {torch.float32: 2, torch.bfloat16: 1, torch.float16: 0}


def _reference(lib, x: torch.Tensor, eps: float) -> torch.Tensor:
    """Output of the existing entry point, with a torch-allocated workspace."""
    batch, rows, cols = x.shape
    ld = (cols + 7) // 8 * 8
    out = torch.zeros((batch, rows, ld), dtype=torch.float16, device=x.device)
    ws = torch.empty(lib.gns_normalize_workspace_size(batch, rows, cols), dtype=torch.uint8, device=x.device)
    rc = lib.gns_frobenius_normalize(CODES[x.dtype], batch, rows, cols, x.data_ptr(), x.stride(0), x.stride(1),
                                     out.data_ptr(), ld, eps, ws.data_ptr(), ws.numel(),
                                     torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _native.last_error()
    return out[:, :, :cols]


def _no_alloc(lib, x: torch.Tensor, eps: float) -> torch.Tensor:
    batch, rows, cols = x.shape
    ld = (cols + 7) // 8 * 8
    out = torch.zeros((batch, rows, ld), dtype=torch.float16, device=x.device)
    rc = lib.gns_frobenius_normalize_noalloc(CODES[x.dtype], batch, rows, cols, x.data_ptr(), x.stride(0),
                                             x.stride(1), out.data_ptr(), ld, eps,
                                             torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _native.last_error()
    return out[:, :, :cols]


def test_no_alloc_normalize_matches_workspace_entry_point(cuda_device):
    lib = _native.load()
    gen = torch.Generator(device=cuda_device).manual_seed(2024)
    cases = [
        (torch.randn((64, 1024, 4096), generator=gen, device=cuda_device) * 1e-2).to(torch.bfloat16),
        torch.randn((3, 200, 72), generator=gen, device=cuda_device),
    ]
    for x in cases:  # two calls in a row through the shared scratch
        got = _no_alloc(lib, x, 1e-7)
        want = _reference(lib, x, 1e-7)
        torch.cuda.synchronize(cuda_device)
        # Same kernel, same partition, same summation order: identical bits.
        torch.testing.assert_close(got, want, rtol=0, atol=0)
        norms = got.float().flatten(1).norm(dim=1)
        torch.testing.assert_close(norms, torch.ones_like(norms), rtol=2e-3, atol=0)


def test_no_alloc_normalize_allocates_nothing(cuda_device):
    lib = _native.load()
    gen = torch.Generator(device=cuda_device).manual_seed(7)
    x = torch.randn((8, 256, 512), generator=gen, device=cuda_device)
    out = torch.zeros((8, 256, 512), dtype=torch.float16, device=cuda_device)
    stream = torch.cuda.current_stream().cuda_stream

    def call() -> None:
        rc = lib.gns_frobenius_normalize_noalloc(CODES[x.dtype], 8, 256, 512, x.data_ptr(), x.stride(0),
                                                 x.stride(1), out.data_ptr(), 512, 1e-7, stream)
        assert rc == 0, _native.last_error()

    call()  # the first call on a device loads the module
    torch.cuda.synchronize(cuda_device)
    free_before, _ = torch.cuda.mem_get_info(cuda_device)
    for _ in range(20):
        call()
    torch.cuda.synchronize(cuda_device)
    free_after, _ = torch.cuda.mem_get_info(cuda_device)
    assert free_after == free_before


def test_no_alloc_normalize_serves_batches_up_to_its_limit(cuda_device):
    lib = _native.load()
    gen = torch.Generator(device=cuda_device).manual_seed(11)
    x = torch.randn((8192, 4, 8), generator=gen, device=cuda_device)
    got = _no_alloc(lib, x, 1e-7)
    want = _reference(lib, x, 1e-7)
    torch.cuda.synchronize(cuda_device)
    torch.testing.assert_close(got, want, rtol=0, atol=0)


def test_no_alloc_normalize_rejects_batches_beyond_its_scratch(cuda_device):
    lib = _native.load()
    rows, cols = 4, 8
    for batch in (8193, 20000):
        rc = lib.gns_frobenius_normalize_noalloc(F16, batch, rows, cols, 16, rows * cols, cols, 16, cols, 1e-7,
                                                 torch.cuda.current_stream().cuda_stream)
        assert rc == -6  # GNS_ERR_UNSUPPORTED, before touching the pointers
        assert "8192" in _native.last_error()
