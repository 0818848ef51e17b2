"""GGUF files and the loader hook (odiengine_b200/gguf.py,
CUDABackend::upload_model).

CPU: a tiny Llama model written by odiengine_b200.gguf is read back by its
own reader and by the reference's parser (src/format/gguf_parser.cpp,
compiled unmodified into the adapter library), with identical metadata,
tensor types, dims and bytes; malformed files are refused by both.
GPU: load_llama uploads every weight once (the stacked Q|K|V and gate|up
blocks unpack to exactly the file's block rows) and the decode step built
on it matches the float64 oracle; CUDABackend::upload_model uploads every
quantized weight of the file once and matmul on the file's own views then
uploads nothing more and matches the oracle product.
"""
import ctypes
import os

import numpy as np
import pytest

import oracle as O
from test_backend_adapter import ADAPTER, BACKEND_CUDA, Backend, _shp, need_adapter

U24 = 2.0 ** -24


def _cfg(ctx=64):
    from odiengine_b200.decode import LlamaConfig

    return LlamaConfig(layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=300, ctx=ctx,
                       act_mode=0)


def _host_model(cfg, seed=3):
    """Host tensors of a tiny model, quantized weights as GGUF blocks (the
    oracle's quantizers), with the reference's tensor names."""
    E, F, H, KV, hd = cfg.hidden, cfg.ffn, cfg.heads, cfg.kv_heads, cfg.head_dim
    rng = np.random.default_rng(seed)
    q = lambda dt, N, K, s: np.ascontiguousarray(O.quantize(dt, O.seeded_weights(N, K, seed=s)))
    h = {"token_embd.weight": rng.standard_normal((cfg.vocab, E)).astype(np.float32)}
    s = 100 * seed
    for l in range(cfg.layers):
        p = f"blk.{l}."
        h[p + "attn_norm.weight"] = (1 + 0.02 * rng.standard_normal(E)).astype(np.float32)
        h[p + "attn_q.weight"] = q(cfg.attn_dtype, H * hd, E, s + 1)
        h[p + "attn_k.weight"] = q(cfg.attn_dtype, KV * hd, E, s + 2)
        h[p + "attn_v.weight"] = q(cfg.attn_dtype, KV * hd, E, s + 3)
        h[p + "attn_output.weight"] = q(cfg.attn_dtype, E, H * hd, s + 4)
        h[p + "ffn_norm.weight"] = (1 + 0.02 * rng.standard_normal(E)).astype(np.float32)
        h[p + "ffn_gate.weight"] = q(cfg.attn_dtype, F, E, s + 5)
        h[p + "ffn_up.weight"] = q(cfg.attn_dtype, F, E, s + 6)
        h[p + "ffn_down.weight"] = q(cfg.down_dtype, E, F, s + 7)
        s += 10
    h["output_norm.weight"] = (1 + 0.02 * rng.standard_normal(E)).astype(np.float32)
    h["output.weight"] = q(cfg.down_dtype, cfg.vocab, E, s + 8)
    return h


@pytest.fixture(scope="module")
def tiny_file(tmp_path_factory):
    from odiengine_b200 import gguf

    cfg = _cfg()
    host = _host_model(cfg)
    path = str(tmp_path_factory.mktemp("gguf") / "tiny.gguf")
    gguf.write_llama(path, cfg, host)
    return cfg, host, path


# --------------------------------------------------------------------------
# CPU
# --------------------------------------------------------------------------
def test_roundtrip_own_reader(tiny_file):
    from odiengine_b200 import gguf

    cfg, host, path = tiny_file
    with gguf.GGUFFile(path) as f:
        assert f.version == 3
        assert f.metadata["general.architecture"] == "llama"
        assert f.metadata["llama.block_count"] == cfg.layers
        assert len(f.metadata["tokenizer.ggml.tokens"]) == cfg.vocab
        assert set(f.names) == set(host)
        for name, arr in host.items():
            assert np.array_equal(f.tensor(name), np.frombuffer(arr.tobytes(), np.uint8)), name
            assert (f.data_start + f.tensors[name].offset) % 32 == 0
        assert f.tensors["blk.0.attn_k.weight"].dims == (cfg.hidden, cfg.kv_heads * cfg.head_dim)
        got = gguf.llama_config(f)
    for k in ("layers", "hidden", "heads", "kv_heads", "head_dim", "ffn", "vocab", "attn_dtype", "down_dtype"):
        assert getattr(got, k) == getattr(cfg, k), k


def test_reference_parser_reads_the_file(tiny_file):
    """The reference's own GGUFFile (gguf_parser.cpp) opens the file and
    returns views with the written dtype, dims and bytes."""
    need_adapter()
    cfg, host, path = tiny_file
    L = Backend.lib()
    f = L.odi_be_gguf_open(path.encode())
    assert f, L.odi_be_last_error()
    try:
        assert L.odi_be_gguf_tensor_count(f) == len(host)
        for name, arr in host.items():
            data, dt, nd = ctypes.c_void_p(), ctypes.c_int(), ctypes.c_int()
            shape = (ctypes.c_int64 * 4)()
            assert L.odi_be_gguf_tensor(f, name.encode(), ctypes.byref(data), ctypes.byref(dt), ctypes.byref(nd),
                                        shape) == 0
            got = np.ctypeslib.as_array((ctypes.c_uint8 * arr.nbytes).from_address(data.value))
            assert np.array_equal(got, np.frombuffer(arr.tobytes(), np.uint8)), name
            if name.endswith("norm.weight"):
                assert dt.value == 0 and nd.value == 1
            elif name != "token_embd.weight":
                want = cfg.down_dtype if ("ffn_down" in name or name == "output.weight") else cfg.attn_dtype
                assert dt.value == want and nd.value == 2, name
        assert L.odi_be_gguf_tensor(f, b"no.such.tensor", ctypes.byref(ctypes.c_void_p()),
                                    ctypes.byref(ctypes.c_int()), ctypes.byref(ctypes.c_int()),
                                    (ctypes.c_int64 * 4)()) != 0
    finally:
        L.odi_be_gguf_close(f)


@pytest.mark.parametrize("damage", ["magic", "truncated", "version"])
def test_malformed_files_refused(tiny_file, tmp_path, damage):
    from odiengine_b200 import gguf

    _, _, path = tiny_file
    raw = bytearray(open(path, "rb").read())
    if damage == "magic":
        raw[0:4] = b"GGUG"
    elif damage == "version":
        raw[4:8] = (7).to_bytes(4, "little")
    else:
        raw = raw[:200]
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(bytes(raw))
    with pytest.raises(ValueError):
        gguf.GGUFFile(str(bad))
    if os.path.exists(ADAPTER):  # header reads are bounds-checked there too (gguf_parser.cpp:243-256)
        L = Backend.lib()
        assert not L.odi_be_gguf_open(str(bad).encode())


# --------------------------------------------------------------------------
# GPU
# --------------------------------------------------------------------------
def _flat(a):
    return np.frombuffer(np.ascontiguousarray(a).tobytes(), np.uint8)


def _oracle_from_host(cfg, host):
    def deq(name, dt, N, K):
        return O.dequantize(dt, host[name], N, K).astype(np.float64)

    E, F, H, KV, hd = cfg.hidden, cfg.ffn, cfg.heads, cfg.kv_heads, cfg.head_dim
    W = {"token_embd": host["token_embd.weight"].astype(np.float64), "out_norm": host["output_norm.weight"],
         "output": deq("output.weight", cfg.down_dtype, cfg.vocab, E)}
    for l in range(cfg.layers):
        p = f"blk.{l}."
        W[f"attn_norm.{l}"] = host[p + "attn_norm.weight"]
        W[f"ffn_norm.{l}"] = host[p + "ffn_norm.weight"]
        W[f"wqkv.{l}"] = np.concatenate([deq(p + "attn_q.weight", cfg.attn_dtype, H * hd, E),
                                         deq(p + "attn_k.weight", cfg.attn_dtype, KV * hd, E),
                                         deq(p + "attn_v.weight", cfg.attn_dtype, KV * hd, E)])
        W[f"wo.{l}"] = deq(p + "attn_output.weight", cfg.attn_dtype, E, H * hd)
        W[f"wgu.{l}"] = np.concatenate([deq(p + "ffn_gate.weight", cfg.attn_dtype, F, E),
                                        deq(p + "ffn_up.weight", cfg.attn_dtype, F, E)])
        W[f"wdown.{l}"] = deq(p + "ffn_down.weight", cfg.down_dtype, E, F)
    return W


@pytest.mark.gpu
def test_load_llama_uploads_blocks_and_decodes(cuda_lib, tiny_file):
    from odiengine_b200 import gguf
    from odiengine_b200.decode import DecodeModel, gate_up_order
    from oracle.llama import LlamaRef

    cfg, host, path = tiny_file
    cfg2, mw = gguf.load_llama(path)
    assert (cfg2.layers, cfg2.hidden, cfg2.vocab, cfg2.ctx) == (cfg.layers, cfg.hidden, cfg.vocab, cfg.ctx)
    # the stacked weights hold exactly the file's block rows, in order
    for l, lw in enumerate(mw.layers):
        p = f"blk.{l}."
        got = cuda_lib.unpack(lw.wqkv.dtype, lw.wqkv.tiled, lw.wqkv.N, lw.wqkv.K).cpu().numpy().ravel()
        want = np.concatenate([_flat(host[p + n]) for n in ("attn_q.weight", "attn_k.weight", "attn_v.weight")])
        assert np.array_equal(got, want)
        got = cuda_lib.unpack(lw.wgu.dtype, lw.wgu.tiled, lw.wgu.N, lw.wgu.K).cpu().numpy().ravel()
        want = np.concatenate([_flat(host[p + n]) for n in ("ffn_gate.weight", "ffn_up.weight")])
        assert mw.gu_interleaved  # gate and up rows interleaved by 32 in every 64-row tile
        want = want.reshape(2 * cfg.ffn, -1)[gate_up_order(cfg.ffn)].ravel()
        assert np.array_equal(got, want)
        got = cuda_lib.unpack(lw.wdown.dtype, lw.wdown.tiled, lw.wdown.N, lw.wdown.K).cpu().numpy().ravel()
        assert np.array_equal(got, _flat(host[p + "ffn_down.weight"]))
    assert np.array_equal(mw.token_embd.cpu().numpy(), host["token_embd.weight"])
    # the decode step on the loaded model against the float64 oracle (Q8 activations: 6e-2 of the logit scale)
    tol = 6e-2
    dm = DecodeModel(cfg2, mw)
    ref = LlamaRef(cfg2, _oracle_from_host(cfg, host))
    prompt = [5, 17, 299, 3]
    dm.prefill(prompt[:-1])
    for p, t in enumerate(prompt[:-1]):
        ref.step(t, p)
    dm.reset(prompt[-1], len(prompt) - 1)
    token, pos = prompt[-1], len(prompt) - 1
    for _ in range(5):
        lr = ref.step(token, pos)
        got = dm.generate(1)[0]
        lg = dm.logits.cpu().numpy().astype(np.float64)
        scale = np.abs(lr).max()
        assert (np.abs(lg - lr) <= tol * scale).all(), np.abs(lg - lr).max() / scale
        top2 = np.sort(lr)[-2:]
        if top2[1] - top2[0] > 2 * tol * scale:
            assert got == int(np.argmax(lr))
        token, pos = got, pos + 1
    assert dm.status() == 0


@pytest.mark.gpu
def test_upload_model_hook(cuda_lib, tiny_file):
    """CUDABackend::upload_model on the reference's GGUFFile: every quantized
    weight uploaded once; matmul on the file's own views then uploads
    nothing and gives the oracle's product (fp32 activations: twice the
    fp32 reordering bound)."""
    need_adapter()
    cfg, host, path = tiny_file
    L = Backend.lib()
    f = L.odi_be_gguf_open(path.encode())
    assert f, L.odi_be_last_error()
    be = Backend(BACKEND_CUDA, act_mode=1)
    try:
        n = ctypes.c_int64(-1)
        assert L.odi_be_upload_model(be.h, f, ctypes.byref(n)) == 0, L.odi_be_last_error()
        n_quant = 7 * cfg.layers + 1
        assert n.value == n_quant and be.cached_weights() == n_quant
        assert L.odi_be_upload_model(be.h, f, ctypes.byref(n)) == 0 and n.value == 0
        for name, dt, N, K in (("blk.1.ffn_down.weight", cfg.down_dtype, cfg.hidden, cfg.ffn),
                               ("blk.0.attn_k.weight", cfg.attn_dtype, cfg.kv_heads * cfg.head_dim, cfg.hidden)):
            data, dtc, nd = ctypes.c_void_p(), ctypes.c_int(), ctypes.c_int()
            shape = (ctypes.c_int64 * 4)()
            assert L.odi_be_gguf_tensor(f, name.encode(), ctypes.byref(data), ctypes.byref(dtc), ctypes.byref(nd),
                                        shape) == 0
            assert (dtc.value, nd.value, shape[0], shape[1]) == (dt, 2, K, N)
            x = O.seeded_acts(3, K, seed=11)
            y = np.full((3, N), np.nan, np.float32)
            rc = L.odi_be_matmul(be.h, y.ctypes.data, 2, _shp(y.shape), x.ctypes.data, 0, 2, _shp(x.shape),
                                 data.value, dt, 2, _shp((K, N)))
            assert rc == 0, L.odi_be_last_error()
            assert be.cached_weights() == n_quant  # found resident: no upload
            b = host[name]
            ref = O.matmul_ref(dt, x, b, N)
            assert (np.abs(y.astype(np.float64) - ref) <= 2.0 * O.fp32_bound(dt, x, b, N)).all()
    finally:
        be.close()
        L.odi_be_gguf_close(f)


@pytest.mark.gpu
def test_cpp_decoder_from_gguf_matches_decode_model(cuda_lib, tiny_file):
    """CUDABackend::create_decoder on the reference's GGUFFile (Q|K|V stacked
    and gate|up interleaved on the host, each uploaded once; the decode step
    driven from C++, one graph replay per token) gives DecodeModel's tokens
    and logits on the same file bit for bit: same kernels, same order, same
    weight layout."""
    from odiengine_b200 import gguf
    from odiengine_b200.decode import DecodeModel

    need_adapter()
    cfg, host, path = tiny_file
    L = Backend.lib()
    f = L.odi_be_gguf_open(path.encode())
    assert f, L.odi_be_last_error()
    be = Backend(BACKEND_CUDA)
    dec = None
    try:
        dec = L.odi_be_decoder_from_gguf(be.h, f, 0, 64)
        assert dec, L.odi_be_last_error()
        fields = (ctypes.c_int * 8)()
        L.odi_be_decoder_config(dec, fields)
        assert list(fields) == [cfg.layers, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn, cfg.vocab,
                                cfg.ctx]
        prompt = [5, 17, 299, 3, 42]
        n = 6
        # C++: the prompt into the cache, then n greedy steps from its last token
        assert L.odi_be_decoder_reset(dec, prompt[0], 0, 1) == 0, L.odi_be_last_error()
        pa = (ctypes.c_int32 * (len(prompt) - 1))(*prompt[:-1])
        assert L.odi_be_decoder_prefill(dec, pa, len(prompt) - 1, 0) == 0, L.odi_be_last_error()
        assert L.odi_be_decoder_reset(dec, prompt[-1], len(prompt) - 1, 0) == 0
        out = (ctypes.c_int32 * n)()
        assert L.odi_be_decoder_generate(dec, n, out) == 0, L.odi_be_last_error()
        logits = np.zeros(cfg.vocab, np.float32)
        assert L.odi_be_decoder_logits(dec, logits.ctypes.data) == 0
        # Python: load_llama + DecodeModel, the same sequence
        cfg2, mw = gguf.load_llama(path)
        dm = DecodeModel(cfg2, mw)
        dm.prefill(prompt[:-1])
        dm.reset(prompt[-1], len(prompt) - 1)
        want = dm.generate(n)
        assert list(out) == want
        assert np.array_equal(logits.view(np.uint32), dm.logits.cpu().numpy().view(np.uint32))
        ms = ctypes.c_float()
        assert L.odi_be_decoder_time(dec, 4, ctypes.byref(ms)) == 0 and ms.value > 0
    finally:
        if dec:
            L.odi_be_decoder_free(dec)
        be.close()
        L.odi_be_gguf_close(f)
