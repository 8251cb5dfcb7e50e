"""The allocation-free gate/up entry point, called through the C ABI.

Some callers of this library cannot allocate device memory for a workspace: a serving process that
has handed the GPU's memory to its own pool at start-up, or a plugin host that passes only its input
and output buffers.  ``reax_gate_up_i8_noalloc`` serves them with scratch held in a static device
array.  This test checks that it returns, on two calls in a row, exactly what the workspace entry
point ``reax_gate_up_i8`` returns for the same inputs (INT8 path: bit-identical, the tolerance every
INT8 test here uses).  The file is named so that pytest collects it last.
"""
import pytest
import torch

from tests import helpers as H

pytestmark = pytest.mark.gpu


def _call_both(M, K, Hh, KH=0):
    from reax_engine_runtime_v3_b200 import _native
    from reax_engine_runtime_v3_b200.reaxv2.gate_up import quantize_rows
    lib = _native.load()
    g = H.gen(9000 + M + K + Hh + KH)
    x = H.activations(g, M, K).cuda()
    bank = H.bank_to(H.int8_bank(g, K, Hh, KH=KH, centered=KH > 0, bias=True), "cuda")
    low, high, scales = quantize_rows(x, bank)
    N2, KL = 2 * Hh, low.shape[1]
    stream = _native.stream_handle()
    ws = torch.zeros(lib.reax_workspace_bytes(-1), dtype=torch.uint8, device="cuda")
    want = torch.empty(M, Hh, dtype=torch.bfloat16, device="cuda")
    hp = high.data_ptr() if KH else None
    whp = bank.high_weight.data_ptr() if KH else None
    _native.check(lib.reax_gate_up_i8(low.data_ptr(), bank.low_weight.data_ptr(), hp, whp, scales.data_ptr(),
                                      bank.scales.data_ptr(), bank.bias.data_ptr(), want.data_ptr(), M, N2, KL, KH,
                                      Hh, ws.data_ptr(), ws.numel(), stream))
    outs = []
    for _ in range(2):
        got = torch.empty(M, Hh, dtype=torch.bfloat16, device="cuda")
        _native.check(lib.reax_gate_up_i8_noalloc(low.data_ptr(), bank.low_weight.data_ptr(), hp, whp,
                                                  scales.data_ptr(), bank.scales.data_ptr(), bank.bias.data_ptr(),
                                                  got.data_ptr(), M, N2, KL, KH, Hh, stream))
        outs.append(got)
        # the call's own status word (bounded waits): clean after each call
        assert _native.noalloc_status() == 0
    torch.cuda.synchronize()
    return want, outs


@pytest.mark.parametrize("M,K,Hh,KH", [
    (64, 4096, 14336, 0),     # decode bucket: weight-major balanced tiles (97 gate rows), whole, no split
    (64, 4096, 1792, 0),      # a rank's shard: weight-major tiles split by K (the partials live in the scratch)
    (1, 1024, 2816, 0),       # single token
    (300, 1024, 4096, 0),     # token-major: 96 tiles, all split, re-planned for the scratch's CTA cap
    (300, 1024, 5504, 0),     # token-major: 129 tiles, re-planned as whole tiles plus a split remainder
    (200, 2560, 1024, 128),   # BF16 outlier columns: whole tiles only
])
def test_noalloc_matches_workspace_entry_point_twice(M, K, Hh, KH):
    want, outs = _call_both(M, K, Hh, KH)
    for got in outs:
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))


def test_noalloc_rejects_bad_shapes_with_a_message():
    from reax_engine_runtime_v3_b200 import _native
    lib = _native.load()
    rc = lib.reax_gate_up_i8_noalloc(None, None, None, None, None, None, None, None, 16, 300, 128, 0, 150,
                                     _native.stream_handle())
    assert rc == 1 and b"N2" in lib.reax_last_error()


def test_noalloc_status_word_reports_an_expired_wait():
    """The allocation-free entry's status word is readable: a self-test wait with a short limit on a
    barrier nothing arrives on records its bit there, reax_noalloc_status reports it and clears it, and
    the next allocation-free call starts clean."""
    from reax_engine_runtime_v3_b200 import _native
    lib = _native.load()
    _native.check(lib.reax_selftest_wait(None, 200000, _native.stream_handle()))
    assert _native.noalloc_status(clear=True) & 0x20
    assert _native.noalloc_status() == 0
    want, outs = _call_both(8, 1024, 2816)
    for got in outs:
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))
