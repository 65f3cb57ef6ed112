"""The dump-state reset of cleared slots (``clear_dump_slots``, C ABI
``aspire_clear_dump_slots``) against the restatement of the reference's
LMBackendBase._clear_variant_slot_state (oracle/dump_state.py): the slots'
dump rows, the LSE rows of their last queries and their mode flags, bit-exact,
for the fp16 first/last dump and the fp32 last-token dump; an out-of-range
slot id is reported and skipped."""

import pytest
import torch

from aspire_b200 import _capi
from aspire_b200.kv_ops import clear_dump_slots
from oracle import dump_state as oracle_dump

pytestmark = pytest.mark.gpu


def _state(dev, B, H, slots, stride, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    dump = (torch.randn(B * H * slots * stride, generator=g) * 9).to(dtype)
    q_lens = torch.randint(1, 10, (B,), generator=g)
    qo = torch.zeros(B + 1, dtype=torch.int32)
    qo[1:] = torch.cumsum(q_lens, 0).to(torch.int32)
    lse = torch.randn(int(qo[-1]) + 3, H, generator=g).float()
    flags = torch.zeros(B, dtype=torch.int32)
    return dump, lse, qo, flags


@pytest.mark.parametrize("dtype,H,slots,stride", [(torch.float16, 16, 2, 1040), (torch.float32, 16, 1, 2053),
                                                 (torch.float16, 5, 2, 1041)],
                         ids=["f16_first_last", "f32_last_token_odd_stride", "f16_unaligned_rows"])
def test_clear_dump_slots_matches_reference(cuda_device, dtype, H, slots, stride):
    """Rows of 5 x 2 x 1041 fp16 values start off the 16-byte grid, so the
    scalar fill path runs too."""
    dev = cuda_device
    B = 6
    dump, lse, qo, flags = _state(dev, B, H, slots, stride, dtype, seed=slots)
    slot_ids = torch.tensor([1, 4, 5], dtype=torch.int32)
    d_dev, l_dev, q_dev, f_dev = dump.to(dev), lse.to(dev), qo.to(dev), flags.to(dev)
    clear_dump_slots(d_dev, slot_ids.to(dev), H, slots, stride, lse_buffer=l_dev, qo_indptr=q_dev,
                     mode_flags=f_dev)
    torch.cuda.synchronize()
    oracle_dump.clear_variant_slot_state(dump, lse, qo, flags, slot_ids, num_heads=H, dump_slots=slots,
                                         kv_stride=stride)
    assert torch.equal(d_dev.cpu(), dump)
    assert torch.equal(l_dev.cpu(), lse)
    assert torch.equal(f_dev.cpu(), flags)
    rows = dump.view(B, -1)
    assert bool(torch.isinf(rows[4]).all()) and not bool(torch.isinf(rows[0]).any())


def test_clear_dump_slots_reports_a_bad_slot(cuda_device):
    dev = cuda_device
    B, H, stride = 4, 8, 512
    dump, lse, qo, flags = _state(dev, B, H, 2, stride, torch.float16, seed=7)
    d_dev = dump.to(dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    clear_dump_slots(d_dev, torch.tensor([2, 9], dtype=torch.int32, device=dev), H, 2, stride, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & _capi.STATUS_BAD_ROW
    expect = dump.clone()
    expect.view(B, -1)[2] = float("-inf")
    assert torch.equal(d_dev.cpu(), expect)


@pytest.mark.parametrize("case", ["f16_first_last", "f32_last_token"])
def test_clear_dump_slots_matches_reference_fixture(cuda_device, golden_dir, case):
    """Against the reference's own _clear_variant_slot_state run on CPU
    (tests/golden/dump_state.pt)."""
    dev = cuda_device
    g = torch.load(golden_dir / "dump_state.pt", weights_only=False)[case]
    p = g["params"]
    d, lse, qo, flags = (g["before"][k].to(dev) for k in ("dump", "lse", "qo_indptr", "mode_flags"))
    clear_dump_slots(d, g["slot_ids"].to(dev), p["H"], p["slots"], p["kv_stride"], lse_buffer=lse, qo_indptr=qo,
                     mode_flags=flags)
    torch.cuda.synchronize()
    assert torch.equal(d.cpu(), g["after"]["dump"])
    assert torch.equal(lse.cpu(), g["after"]["lse"])
    assert torch.equal(flags.cpu(), g["after"]["mode_flags"])
