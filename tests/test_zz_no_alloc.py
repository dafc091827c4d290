"""The allocation-free LM-head argmax entry point, called through the C ABI.

tempo_lm_head_argmax_noalloc serves callers that may not allocate device memory (a plugin host that owns every device
byte, or a loop that cannot afford cudaMalloc/cudaFree): it keeps the partials between its two kernels in an array
compiled into the library instead of a caller buffer. This test holds it to the allocating path (tempo_gemm in argmax
mode plus tempo_argmax_finish with caller-allocated partials) on calls in a row with fewer rows each time, so every
call after the first runs over the previous call's leftover contents: 300 and 17 rows take the tensor-core argmax
GEMM, 8 rows and 1 row the CUDA-core GEMV argmax kernel, which writes the partials with its own kernel. It also
checks that sizes past the array's limits are refused. The tokens must be identical: both paths run the same
kernels. The file is named to be collected last.
"""

from __future__ import annotations

import ctypes

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _allocating_path(hidden, embedding):
    from tempo_compiler_b200 import ops
    rows, vocab = hidden.shape[0], embedding.shape[0]
    tiles = (vocab + 255) // 256
    part_val = torch.empty((rows, tiles), dtype=torch.float32, device="cuda")
    part_idx = torch.empty((rows, tiles), dtype=torch.int32, device="cuda")
    ids = torch.empty(rows, dtype=torch.int32, device="cuda")
    ops.gemm_argmax(hidden, embedding, part_val, part_idx)
    ops.argmax_finish(part_val, part_idx, ids)
    return ids


def test_noalloc_lm_head_argmax_matches_the_allocating_path() -> None:
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from tempo_compiler_b200 import lib
    library = lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    width, vocab = 768, 50257
    generator = torch.Generator(device="cuda").manual_seed(77)
    embedding = (torch.randn((vocab, width), generator=generator, device="cuda") * 0.02).to(torch.bfloat16)
    for rows in (300, 17, 8, 1):
        hidden = torch.randn((rows, width), generator=generator, device="cuda").to(torch.bfloat16)
        ids = torch.full((rows,), -1, dtype=torch.int32, device="cuda")
        status = library.tempo_lm_head_argmax_noalloc(hidden.data_ptr(), width, embedding.data_ptr(), width, rows,
                                                      vocab, width, ids.data_ptr(), stream)
        assert status == lib.OK, lib.last_error()
        expected = _allocating_path(hidden, embedding)
        torch.cuda.synchronize()
        assert torch.equal(ids, expected)
        assert int(ids.min()) >= 0 and int(ids.max()) < vocab

    too_many = torch.empty((1025, width), dtype=torch.bfloat16, device="cuda")
    out = torch.empty(1025, dtype=torch.int32, device="cuda")
    status = library.tempo_lm_head_argmax_noalloc(too_many.data_ptr(), width, embedding.data_ptr(), width, 1025, vocab,
                                                  width, out.data_ptr(), stream)
    assert status == lib.ERR_VALUE and "1024" in lib.last_error()
    status = library.tempo_lm_head_argmax_noalloc(too_many.data_ptr(), width, embedding.data_ptr(), width, 4, 65537,
                                                  width, out.data_ptr(), stream)
    assert status == lib.ERR_VALUE and "65536" in lib.last_error()
    torch.cuda.synchronize()
    code = ctypes.c_int32()
    assert library.tempo_watchdog(ctypes.byref(code)) == lib.OK and code.value == 0
