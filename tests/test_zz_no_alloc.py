"""The no-allocation text encoder entry point against the allocating one.

jb_encode_text_device_noalloc serves callers that must not allocate device
memory (cudaMalloc/cudaFree synchronise the device; a process whose device
memory is reserved by another runtime's pool has none to give).  Its scratch
is a 64 MiB array inside the library, shared by every call on a device.
This file is collected last on purpose: it must pass both on its own in a
fresh process and after every other test.  The no-allocation call runs the
same kernels in the same order as the allocating one, so the two are
compared bit for bit.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TOL = 2e-3   # the bf16 / int8 embedding bar used by the encoder parity tests
COS = 0.9999


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from jammi_b200 import _lib
    return _lib


def _model(fmt):
    from jammi_b200 import Bert
    from jammi_b200.synthetic import bert_weights
    cfg = dict(hidden_size=768, num_hidden_layers=2, num_attention_heads=12, intermediate_size=3072,
               vocab_size=30522, max_position_embeddings=512, type_vocab_size=2,
               layer_norm_eps=1e-12, model_type="bert")
    return Bert.from_weights(bert_weights(cfg, seed=77), cfg, device=0, fmt=fmt)


def _batch(seed, batch, seq):
    from jammi_b200.synthetic import token_batch, uniform_lengths
    rng = np.random.default_rng(seed)
    lens = uniform_lengths(rng, batch, 1, seq)
    ids = token_batch(rng, lens, seq)
    return (torch.from_numpy(ids.astype(np.int32)).cuda(),
            torch.from_numpy(lens.astype(np.int32)).cuda())


def _noalloc(lib, model, ids, lens, batch, seq, out):
    return lib.lib().jb_encode_text_device_noalloc(
        model.handle, ids.data_ptr(), lens.data_ptr(), batch, seq, lib.POOL_MEAN, out.data_ptr(),
        torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("fmt", ["bf16", "int8"])
def test_noalloc_matches_allocating_entry_point(lib, fmt):
    """Two calls in a row, each against jb_encode_text_device on the same
    inputs: the two entry points run the same kernels in the same order on
    the same data, so the embeddings are equal bit for bit."""
    model = _model(fmt)
    L = lib.lib()
    s = torch.cuda.current_stream().cuda_stream
    for call, (batch, seq) in enumerate([(8, 128), (13, 96)]):
        ids, lens = _batch(100 + call, batch, seq)
        ref = torch.empty((batch, 768), device="cuda")
        got = torch.full((batch, 768), float("nan"), device="cuda")
        lib.check(L.jb_encode_text_device(model.handle, ids.data_ptr(), lens.data_ptr(), batch, seq,
                                          lib.POOL_MEAN, ref.data_ptr(), s))
        lib.check(_noalloc(lib, model, ids, lens, batch, seq, got))
        model.sync(torch.cuda.current_stream())
        assert torch.isfinite(got).all()
        assert torch.equal(got, ref), (got - ref).abs().max().item()
    model.close()


@pytest.mark.parametrize("fmt", ["bf16", "int8"])
def test_noalloc_only_handle_allocates_nothing(lib, fmt):
    """A handle that only ever uses the no-allocation entry point: after one
    warm-up call of a shape (which may load kernel code), a second call of
    that shape leaves the device's free memory exactly where it was, and its
    output equals the allocating entry point's, computed afterwards."""
    model = _model(fmt)
    L = lib.lib()
    batch, seq = 11, 112
    ids, lens = _batch(200, batch, seq)
    got = torch.full((batch, 768), float("nan"), device="cuda")
    ref = torch.empty((batch, 768), device="cuda")
    lib.check(_noalloc(lib, model, ids, lens, batch, seq, got))      # warm-up
    model.sync(torch.cuda.current_stream())
    free0, _ = torch.cuda.mem_get_info()
    got.fill_(float("nan"))
    lib.check(_noalloc(lib, model, ids, lens, batch, seq, got))
    model.sync(torch.cuda.current_stream())
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, f"{free0 - free1} bytes of device memory taken by a no-alloc call"
    lib.check(L.jb_encode_text_device(model.handle, ids.data_ptr(), lens.data_ptr(), batch, seq,
                                      lib.POOL_MEAN, ref.data_ptr(),
                                      torch.cuda.current_stream().cuda_stream))
    model.sync(torch.cuda.current_stream())
    assert torch.equal(got, ref)
    model.close()


def test_noalloc_rejects_requests_above_its_scratch(lib):
    model = _model("bf16")
    L = lib.lib()
    ids, lens = _batch(5, 64, 512)  # ~1.4 GB of scratch for a 768-wide model
    out = torch.empty((64, 768), device="cuda")
    st = _noalloc(lib, model, ids, lens, 64, 512, out)
    assert st == lib.ERR_INVALID
    msg = L.jb_last_error().decode()
    assert "64 MiB" in msg and "scratch" in msg
    model.close()


def test_noalloc_rejects_the_open_clip_text_tower(lib):
    import json
    from conftest import load_golden
    from jammi_b200 import OpenClipText
    w, g = load_golden("small_clip_text.npz")
    model = OpenClipText.from_weights(w, json.loads(bytes(g["config_json"]).decode()), device=0,
                                      fmt="bf16")
    ids = torch.from_numpy(g["ids"].astype(np.int32)).cuda()
    lens = torch.full((ids.shape[0],), ids.shape[1], dtype=torch.int32, device="cuda")
    out = torch.empty((ids.shape[0], 32), device="cuda")
    assert _noalloc(lib, model, ids, lens, ids.shape[0], ids.shape[1], out) == lib.ERR_INVALID
    assert "OpenCLIP text" in lib.lib().jb_last_error().decode()
    model.close()
