"""Failure detection without a GPU fault: every wait inside the kernels is bounded. A wait that runs out records a code
in the caller's device error word, raises the CTA's abort flag and returns; the kernel ends normally and the context
stays usable. The GPU test makes a wait run out on purpose (a barrier nothing completes) through the library's
self-test entry point, checks the recorded status, then runs a regular kernel on the same context. The multi-rank side
(a rank that never joins) is covered on CPU by tests/test_dp.py."""

import pytest
import torch

import oracle
from belt_b200 import _lib
from belt_b200 import decode as dec


def test_selftest_entry_rejects_null_buffers():
    lib = _lib.load()
    assert lib.belt_selftest_bounded_wait(None, None, None) == -1
    assert "null" in lib.belt_last_error().decode()


@pytest.mark.gpu
def test_bounded_wait_runs_out_and_context_survives():
    dev = torch.device("cuda", 0)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    status = torch.zeros(2, dtype=torch.int32, device=dev)
    _lib.call("belt_selftest_bounded_wait", err.data_ptr(), status.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
    torch.cuda.synchronize(dev)
    assert status.tolist() == [2, 1]          # the wait gave up and raised the abort flag
    assert int(err.item()) == 0x1F0           # the code reached the host through the error word
    # the context is still usable: a regular kernel of the library runs and gives the right answer
    seqs = [300, 0, 129]
    sched = dec.make_schedule(len(seqs), dev, num_ctas=4, start_cost=0)
    dec.schedule(sched, torch.tensor(seqs, dtype=torch.int32, device=dev))
    torch.cuda.synchronize(dev)
    _, cta_seg, seg_base = oracle.schedule(seqs, 4, dec.TILE_T)
    assert sched.seg_base.tolist() == seg_base.tolist()
    assert sched.cta_seg.tolist() == cta_seg.tolist()


@pytest.mark.gpu
def test_error_word_surfaces_as_exception():
    dev = torch.device("cuda", 0)
    word = dec.error_word(dev)
    status = torch.zeros(2, dtype=torch.int32, device=dev)
    _lib.call("belt_selftest_bounded_wait", word.data_ptr(), status.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
    with pytest.raises(_lib.BeltError, match="0x1f0"):
        dec.check_device_errors(dev)
    assert int(word.item()) == 0              # check_device_errors clears the word


@pytest.mark.gpu
def test_metadata_builder_raises_on_an_earlier_steps_error():
    """The backend checks the error word without a synchronisation: each build reads the copy of the word that the
    previous build enqueued. A wait that ran out in the step between two builds makes the second build raise."""
    from belt_b200.latent_backend import CommonAttentionMetadata, LatentAttentionMetadataBuilder, LatentKVSpec
    dev = torch.device("cuda", 0)
    seqs = [300, 17]
    B = len(seqs)
    builder = LatentAttentionMetadataBuilder(LatentKVSpec(block_size=16, head_size=1024), ["l0"], device=dev,
                                             max_num_batched_tokens=64)

    def common():
        return CommonAttentionMetadata(query_start_loc=torch.arange(B + 1, dtype=torch.int32, device=dev),
                                       query_start_loc_cpu=torch.arange(B + 1, dtype=torch.int32),
                                       seq_lens=torch.tensor(seqs, dtype=torch.int32, device=dev),
                                       block_table_tensor=torch.zeros(B, 32, dtype=torch.int32, device=dev),
                                       slot_mapping=torch.zeros(B, dtype=torch.int64, device=dev), num_reqs=B,
                                       num_actual_tokens=B, max_query_len=1)
    dec.check_device_errors(dev)                     # start from a clear word
    builder.build(0, common())
    torch.cuda.synchronize(dev)
    builder.build(0, common())                       # clean step: reads a zero word
    word = dec.error_word(dev)
    status = torch.zeros(2, dtype=torch.int32, device=dev)
    _lib.call("belt_selftest_bounded_wait", word.data_ptr(), status.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
    torch.cuda.synchronize(dev)
    builder.build(0, common())                       # its copy of the word is enqueued after the failed wait
    torch.cuda.synchronize(dev)
    with pytest.raises(_lib.BeltError, match="0x1f0"):
        builder.build(0, common())
    torch.cuda.synchronize(dev)
    assert int(word.item()) == 0
    builder.build(0, common())                       # cleared: later steps build again
