"""Kernel classification in the comm/compute split, and the tokenizers."""

import pytest

from build_your_own_distributed_training_b200.data.tokenizer import ByteTokenizer, HFTokenizer, Tokenizer, build_tokenizer
from build_your_own_distributed_training_b200.observability.profiler import is_comm_kernel, is_fused_comm_kernel

# names as the CUDA profiler reports them
PEER_AR = "void dtb::gemm_tcgen05_kernel<256, 6, 1, 1, 6, 1>(CUtensorMap_st, CUtensorMap_st, dtb::GemmArgs)"
SWIGLU = "void dtb::gemm_tcgen05_kernel<256, 6, 0, 0, 5, 1>(CUtensorMap_st, CUtensorMap_st, dtb::GemmArgs)"
ACC = "void dtb::gemm_tcgen05_kernel<256, 6, 1, 1, 2, 1>(CUtensorMap_st, CUtensorMap_st, dtb::GemmArgs)"
PEER_AR_BOOLS = "void dtb::gemm_tcgen05_kernel<256, 6, false, true, 6, true>(CUtensorMap_st, CUtensorMap_st, dtb::GemmArgs)"
ROPE_BOOLS = "void dtb::gemm_tcgen05_kernel<256, 6, false, false, 4, true>(CUtensorMap_st, CUtensorMap_st, dtb::GemmArgs)"


def test_peer_epilogue_gemm_is_fused_not_compute_or_comm():
    assert is_fused_comm_kernel(PEER_AR) and not is_comm_kernel(PEER_AR)
    assert is_fused_comm_kernel(PEER_AR_BOOLS) and not is_fused_comm_kernel(ROPE_BOOLS)
    for name in (SWIGLU, ACC, ROPE_BOOLS):
        assert not is_fused_comm_kernel(name) and not is_comm_kernel(name)


def test_collectives_are_comm():
    for name in ("ncclDevKernel_AllReduce_Sum_f32_RING_LL(ncclDevKernelArgsStorage<4096ul>)",
                 "dtb::comm::peer_all_gather_kernel(dtb::comm::PeerPtrs, long, int, int, int*)",
                 "dtb::comm::dev_barrier_kernel(unsigned int**, int, int, unsigned int, int*)"):
        assert is_comm_kernel(name) and not is_fused_comm_kernel(name)
    assert not is_comm_kernel("dtb::adamw_kernel(float *, const float *)")


def test_byte_tokenizer_round_trip_and_range_check():
    tok = build_tokenizer("")
    assert isinstance(tok, ByteTokenizer) and isinstance(tok, Tokenizer) and tok.vocab_size == 256
    text = "naïve — 2D parallel"
    ids = tok.encode(text)
    assert all(0 <= i < 256 for i in ids) and len(ids) == len(text.encode("utf-8"))
    assert tok.decode(ids) == text
    assert tok.decode(ids[:3]) == "na�"  # a character cut in half
    with pytest.raises(ValueError):
        tok.decode([65, 300])
    assert isinstance(build_tokenizer(None), ByteTokenizer)


def test_hf_tokenizer_is_lazy():
    tok = build_tokenizer("some/model-that-is-not-downloaded")
    assert isinstance(tok, HFTokenizer) and tok._impl is None  # nothing loaded until first use
