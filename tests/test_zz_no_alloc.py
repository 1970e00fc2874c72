"""The scratch-free attention entry point (``mt_attention_decode_noalloc``).

It exists for callers that cannot allocate device memory for the split-K scratch:
real-time audio callbacks that must not block on an allocator (an allocation can
synchronise the device), and plugin or foreign-function hosts with no device allocator of
their own. It keeps its scratch in a fixed array inside the library.

This test calls it through the C ABI twice in a row (the second call sees whatever the
first left in the shared array) and checks each result against the allocating entry
point ``mt_attention_decode`` on identical inputs -- both its default cluster kernel and
its split-K kernel with caller-owned scratch (the same kernel the scratch-free entry point
runs) -- within the tolerance the other GPU tests use, plus the documented rejection of a
request larger than the fixed array.
It is collected last so a failure here cannot hide the rest of the suite, and it builds
everything it needs itself, so it also passes alone in a fresh process.
"""
import numpy as np
import pytest
import torch

from moss_tts._runtime import native, synthetic
from moss_tts._runtime.engine import rope_tables

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2


def _bf16(bits, device):
    a = np.ascontiguousarray(bits, dtype=np.uint16)
    return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).to(device)


def test_noalloc_attention_matches_allocating_entry_point(cuda_device):
    dev = cuda_device
    nq, nkv, max_len, splits = 32, 8, 1024, 18
    stream = torch.cuda.current_stream(dev).cuda_stream
    cos, sin = (t.to(dev) for t in rope_tables(max_len))
    qn = _bf16(synthetic.activation(31, (128,), 0.02), dev) + 1.0
    kn = _bf16(synthetic.activation(32, (128,), 0.02), dev) + 1.0
    qn, kn = qn.to(torch.bfloat16).contiguous(), kn.to(torch.bfloat16).contiguous()
    k_a = _bf16(synthetic.activation(33, (1, nkv, max_len, 128)), dev)
    v_a = _bf16(synthetic.activation(34, (1, nkv, max_len, 128)), dev)
    k_b, v_b, k_c, v_c = k_a.clone(), v_a.clone(), k_a.clone(), v_a.clone()
    partial = torch.empty(nkv * splits * 4 * 128, device=dev)
    lse = torch.empty(nkv * splits * 4, device=dev)
    tickets = torch.zeros(nkv, device=dev, dtype=torch.int32)
    for call, position in enumerate((700, 701)):  # two calls in a row, different inputs
        qkv = _bf16(synthetic.activation(40 + call, (1, (nq + 2 * nkv) * 128)), dev)
        pos = torch.tensor([position], device=dev)
        out_a = torch.empty((1, nq * 128), device=dev, dtype=torch.bfloat16)
        out_b, out_c = torch.empty_like(out_a), torch.empty_like(out_a)
        for flags, out, k, v in ((0, out_a, k_a, v_a), (native.FLAG_REGISTER_PIPELINE, out_c, k_c, v_c)):
            native.call("mt_attention_decode", qkv.data_ptr(), qn.data_ptr(), kn.data_ptr(), cos.data_ptr(),
                        sin.data_ptr(), pos.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                        partial.data_ptr(), lse.data_ptr(), tickets.data_ptr(), 1, nq, nkv, max_len, splits,
                        1e-6, None, flags, stream)
        native.call("mt_attention_decode_noalloc", qkv.data_ptr(), qn.data_ptr(), kn.data_ptr(),
                    cos.data_ptr(), sin.data_ptr(), pos.data_ptr(), k_b.data_ptr(), v_b.data_ptr(),
                    out_b.data_ptr(), 1, nq, nkv, max_len, splits, 1e-6, None, 0, stream)
        torch.cuda.synchronize(dev)
        a, b, c = (o.float().cpu().numpy() for o in (out_a, out_b, out_c))
        err = np.abs(a - b).max()
        print(f"noalloc call {call}: max |cluster - noalloc| = {err:.3g}")
        assert np.all(np.abs(a - b) <= ATOL + RTOL * np.abs(a)), (call, err)
        # the same split-K kernel over caller-owned scratch gives the same bits
        assert np.array_equal(b, c), (call, np.abs(b - c).max())
        assert torch.equal(k_a, k_b) and torch.equal(v_a, v_b) and torch.equal(k_a, k_c)  # same cache rows
        assert float(out_b.float().abs().sum()) > 0.0


def test_noalloc_rejects_requests_beyond_its_fixed_scratch(cuda_device):
    dev = cuda_device
    z = torch.zeros(16, device=dev, dtype=torch.bfloat16)
    pos = torch.zeros(1, device=dev, dtype=torch.long)
    kv = torch.zeros((8, 128, 128), device=dev, dtype=torch.bfloat16)
    # 64 sequences x 8 KV heads x 64 splits x 4 heads x 128 floats is 16 MiB > 1 MiB
    rc = native.library().mt_attention_decode_noalloc(
        z.data_ptr(), z.data_ptr(), z.data_ptr(), z.data_ptr(), z.data_ptr(), pos.data_ptr(), kv.data_ptr(),
        kv.data_ptr(), z.data_ptr(), 64, 32, 8, 128, 64, 1e-6, None, 0,
        torch.cuda.current_stream(dev).cuda_stream)
    assert rc == 2  # cudaErrorMemoryAllocation: larger than the fixed scratch, nothing launched
