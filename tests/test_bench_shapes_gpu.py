"""Parity at the benchmark's own full-size inputs (BASELINE configs 3 and 4).

The bench times the decode kernel on config 3 (B=64, contexts U[512, 29600],
a 131072-block pool) and the tcgen05 prefill + decode kernels on config 4
(prefill contexts U[0, 8192], decode contexts U[256, 16384]).  These tests
build exactly those inputs (``bench.config3_inputs`` / ``config4_inputs``),
run the same calls, and check a seeded subset of requests against the CPU
oracle at the bf16 bound (max-abs 2e-2); every output row must be finite and
no device error may be raised.  The oracle sees a compact copy of only the
checked requests' blocks, so the CPU work stays within seconds.
"""

import pytest
import torch

import bench
from oracle import attention as oatt

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _compact(kc, vc, tables, rows, lens):
    """The checked requests' blocks as a small CPU pool, with tables renumbered."""
    keep, new_tables = [], []
    for r in rows:
        n = -(-lens[r] // 16)
        ids = tables[r, :n].tolist()
        new_tables.append(list(range(len(keep), len(keep) + n)))
        keep.extend(ids)
    idx = torch.tensor(keep, dtype=torch.long, device=kc.device)
    return kc[:, idx].cpu(), vc[:, idx].cpu(), new_tables


def test_config3_bench_inputs_against_oracle(cuda):
    from nano_infer_engine_b200 import ops

    inp = bench.config3_inputs(cuda)
    out = ops.paged_decode(inp["q"], inp["kc"], inp["vc"], 0, inp["tables_d"], inp["lens_d"])
    ops.check_device_errors(cuda)
    assert torch.isfinite(out).all()
    g = torch.Generator().manual_seed(3)
    rows = torch.randperm(64, generator=g)[:8].tolist()
    rows[0] = max(range(64), key=lambda r: inp["lens"][r])  # the longest context is always checked
    kc, vc, tables = _compact(inp["kc"], inp["vc"], inp["tables"], rows, inp["lens"])
    want = oatt.paged_decode(inp["q"][rows].cpu(), kc, vc, tables, [inp["lens"][r] for r in rows], 0)
    torch.testing.assert_close(out[rows].cpu().float(), want.float(), atol=TOL, rtol=0)
    del inp
    torch.cuda.empty_cache()


def test_config4_bench_inputs_against_oracle(cuda):
    from nano_infer_engine_b200 import ops

    inp = bench.config4_inputs(cuda)
    out = torch.full_like(inp["q"], float("nan"))
    bench.config4_prefill(inp, out)
    bench.config4_decode(inp, out)
    ops.check_device_errors(cuda)
    assert torch.isfinite(out).all()  # every row written: 8 x 128 prefill rows + 120 decode rows
    contexts, qlens, lens = inp["contexts"], inp["qlens"], inp["lens"]
    qsl = [0]
    for n in qlens:
        qsl.append(qsl[-1] + n)
    # all 8 prefill segments (the tcgen05 kernel with the split-KV merge)
    pf = list(range(8))
    kc, vc, tables = _compact(inp["kc"], inp["vc"], inp["tables"], pf, lens)
    q_pf = inp["q"][: qsl[8]].cpu()
    want = oatt.varlen_attention(q_pf, kc, vc, tables, contexts[:8], qlens[:8], 0)
    torch.testing.assert_close(out[: qsl[8]].cpu().float(), want.float(), atol=TOL, rtol=0)
    # 16 seeded decode rows, the longest included
    g = torch.Generator().manual_seed(4)
    dec = [8 + i for i in torch.randperm(120, generator=g)[:16].tolist()]
    dec[0] = max(range(8, 128), key=lambda r: lens[r])
    kc, vc, tables = _compact(inp["kc"], inp["vc"], inp["tables"], dec, lens)
    q_dec = inp["q"][[qsl[r] for r in dec]].cpu()
    want = oatt.paged_decode(q_dec, kc, vc, tables, [lens[r] for r in dec], 0)
    torch.testing.assert_close(out[[qsl[r] for r in dec]].cpu().float(), want.float(), atol=TOL, rtol=0)
    del inp
    torch.cuda.empty_cache()
