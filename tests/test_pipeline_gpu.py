"""Drop-in validation under the reference's own runtime (skipped when the
reference is not installed under baseline/_ref).

A random-init bundle of the reference's modules -- a 2-layer w2v-BERT encoder
(relative_key, 64 / 8), a 2-block CTM DiT head, a 2-iteration WaveFitNeXt
latent decoder with its default generator -- goes into the reference's
``TritonModel`` and ``TritonPipeline`` (triton/src/fds_triton/runtime.py:80).
The pipeline runs its own path: per (length, batch) an eager warm-up on a side
stream, then ``torch.cuda.graph`` capture into a shared pool and replay
(``run_chain``, runtime.py:153-177), with 10 s buckets (``separate``,
runtime.py:185-201) and batches of same-bucket windows (``separate_batch``,
runtime.py:203-223). The attention calls the model makes -- the encoder's
``K.encoder_attention`` (model.py:290) and the DiT's ``K.rope_split`` + SDPA
(model.py:319-325) -- are swapped for this library's ops, and the output audio
is compared with the same pipeline running the reference's own ops, on the same
waveforms and the same noise (the pipeline draws it eagerly before each replay;
both runs seed the CUDA generator identically).

``stream_files`` (runtime.py:226-283) runs on two synthetic 120 s 16 kHz
int16 wav files written to a temporary directory: its reader thread, pinned
double buffers, copy stream and writer thread, one graph at the full 6000-frame
window, and the int16 wav files it writes are compared between the two runs.

Bars: our pipeline against the reference's, SNR >= 30 dB on the audio (both
approximate the fp32 model at the fp16 bar; the random-init vocoder amplifies
small latent differences); graph replay against eager, >= 60 dB.
"""

import os
import sys
import types
import wave
from contextlib import contextmanager
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.nn.functional as Fn

import fastdialoguesidon_b200 as F
from oracle import flexrel_oracle as O

pytestmark = pytest.mark.gpu

REF_DIR = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


@pytest.fixture(scope="module")
def ref():
    if not (REF_DIR / "fds_triton").is_dir():
        pytest.skip("reference package not installed under baseline/_ref")
    os.environ.setdefault("FDS_FLEX_NO_COMPILE", "1")
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    from fds_triton import model as M
    from fds_triton import runtime as R
    from fds_triton.reference import modeling as RM
    from fds_triton.reference import wavefit_next as W
    return M, R, RM, W


def _bundle(RM, W, seed=0):
    import transformers

    torch.manual_seed(seed)
    cfg = transformers.Wav2Vec2BertConfig(
        hidden_size=1024, num_attention_heads=16, num_hidden_layers=2, intermediate_size=4096,
        position_embeddings_type="relative_key", left_max_position_embeddings=64,
        right_max_position_embeddings=8, feature_projection_input_dim=160)
    ssl = transformers.Wav2Vec2BertModel(cfg)
    RM.replace_attention_with_flex(ssl)
    latent = 32
    encoder = RM.DialogueEncoder(ssl, latent).cuda().eval()
    head = RM.CTMTransformerHead(latent_size=2 * latent, cond_size=2 * latent + 1024, hidden_size=768,
                                 num_layers=2, num_heads=12)
    ctm = RM.CTMOneStep(head, dict(alpha_t=0.6, sigma_t=0.8, c_skip=0.25, c_out=0.75)).cuda().eval()
    vocoder = W.WaveFitNeXtLatentDecoder(num_iteration=2, latent_dim=latent, sample_rate=24000, latent_rate=50,
                                         n_fft_stft=1024).cuda().eval()
    return types.SimpleNamespace(encoder=encoder, head=head, ctm=ctm, vocoder=vocoder,
                                 latent_mean=torch.zeros(2 * latent, device="cuda"),
                                 latent_std=torch.ones(2 * latent, device="cuda"))


@contextmanager
def _our_attention(M):
    """This library's ops at the model's attention call sites."""
    stash = {}

    def rope_split_stash(qkv, length, heads, cos, sin):  # the call's inputs for the SDPA below
        stash.update(qkv=qkv, length=length, heads=heads, cos=cos, sin=sin)
        dummy = qkv.new_empty(qkv.shape[0], heads * 64)
        return dummy, dummy, dummy

    def attention_ours(q, k, v, *args, **kwargs):  # [B, H, L, 64], as the call site expects
        qkv, length, heads = stash["qkv"], stash["length"], stash["heads"]
        batch = qkv.shape[0] // length
        out = F.rope_attention(qkv, batch, heads, stash["cos"], stash["sin"])
        return out.view(batch, length, heads, 64).transpose(1, 2)

    saved = (M.K.encoder_attention, M.K.rope_split, Fn.scaled_dot_product_attention)
    M.K.encoder_attention = lambda qkv, batch, heads, rel, impl="split": F.encoder_attention(
        qkv, batch, heads, rel, impl)
    M.K.rope_split = rope_split_stash
    Fn.scaled_dot_product_attention = attention_ours
    try:
        yield
    finally:
        M.K.encoder_attention, M.K.rope_split, Fn.scaled_dot_product_attention = saved


def _waves(seconds, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return [torch.randn(int(s * 16000), generator=g, device="cuda") * 0.1 for s in seconds]


def _separate(pipe, waves, seed):
    out = []
    for i, w in enumerate(waves):
        torch.cuda.manual_seed(seed + i)  # the noise run_chain draws before the replay
        out.append(pipe.separate(w))
    return out


def test_pipeline_graphs_and_buckets_with_our_attention(ref):
    M, R, RM, W = ref
    bundle = _bundle(RM, W)
    model = M.TritonModel(bundle, max_seq=R.SEQ)
    waves = _waves([7.3, 15.0, 9.1], seed=1)   # buckets 10 s, 20 s, 10 s (the third replays a graph)
    theirs = _separate(R.TritonPipeline(None, model=model, bucket_seconds=10), waves, seed=100)
    with _our_attention(M):
        pipe = R.TritonPipeline(None, model=model, bucket_seconds=10)
        ours = _separate(pipe, waves, seed=100)
        assert sorted(pipe._graphs) == [(500, 1), (1000, 1)]  # one graph per bucket, captured once
        eager = _separate(R.TritonPipeline(None, model=model, use_graph=False, bucket_seconds=10), waves[:1],
                          seed=100)
    F.check_status()
    for i, (a, b) in enumerate(zip(theirs, ours)):
        assert a.shape == b.shape == (2, waves[i].numel() * 3 // 2)
        snr = O.snr_db(a.float().cpu(), b.float().cpu())
        print(f"window {i}: our attention vs the reference's, {snr:.1f} dB")
        assert snr >= 30.0, (i, snr)
    assert O.snr_db(eager[0].float().cpu(), ours[0].float().cpu()) >= 60.0


def test_separate_batch_with_our_attention(ref):
    M, R, RM, W = ref
    bundle = _bundle(RM, W, seed=1)
    model = M.TritonModel(bundle, max_seq=R.SEQ)
    waves = _waves([12.0, 18.5], seed=2)  # one 20 s bucket, batch 2
    torch.cuda.manual_seed(7)
    theirs = R.TritonPipeline(None, model=model, bucket_seconds=10, max_batch=2).separate_batch(waves)
    with _our_attention(M):
        torch.cuda.manual_seed(7)
        ours = R.TritonPipeline(None, model=model, bucket_seconds=10, max_batch=2).separate_batch(waves)
    F.check_status()
    assert theirs.shape == ours.shape
    snr = O.snr_db(theirs.float().cpu(), ours.float().cpu())
    print(f"separate_batch: our attention vs the reference's, {snr:.1f} dB")
    assert snr >= 30.0, snr


def _write_wav(path, data, rate=16000):
    with wave.open(str(path), "wb") as handle:
        handle.setnchannels(1)
        handle.setsampwidth(2)
        handle.setframerate(rate)
        handle.writeframes(data.astype(np.int16).tobytes())


def _read_wav(path):
    with wave.open(str(path), "rb") as handle:
        return np.frombuffer(handle.readframes(handle.getnframes()), dtype=np.int16)


def test_stream_files_with_our_attention(ref, tmp_path):
    M, R, RM, W = ref
    bundle = _bundle(RM, W, seed=2)
    model = M.TritonModel(bundle, max_seq=R.SEQ)
    rng = np.random.default_rng(3)
    paths = []
    for i in range(2):  # two full 120 s windows, 16 kHz mono int16
        p = tmp_path / f"call{i}.wav"
        _write_wav(p, np.clip(rng.normal(0.0, 3000.0, R.SAMPLES), -32768, 32767))
        paths.append(p)
    outs = {}
    for name in ("theirs", "ours"):
        out_dir = tmp_path / name
        torch.cuda.manual_seed(11)  # the noise run_chain draws before each window
        if name == "ours":
            with _our_attention(M):
                R.stream_files(R.TritonPipeline(None, model=model, bucket_seconds=10), paths, out_dir)
        else:
            R.stream_files(R.TritonPipeline(None, model=model, bucket_seconds=10), paths, out_dir)
        outs[name] = {f.name: _read_wav(f) for f in sorted(out_dir.glob("*.wav"))}
    F.check_status()
    assert sorted(outs["ours"]) == sorted(outs["theirs"]) == [f"call{i}_spk{s}.wav" for i in range(2) for s in (0, 1)]
    for fname, a in outs["theirs"].items():
        b = outs["ours"][fname]
        assert a.shape == b.shape == (R.OUT_SAMPLES,)
        assert np.abs(a).max() > 100, fname  # the audio is not silent at int16 resolution
        snr = O.snr_db(torch.from_numpy(a.astype(np.float32)), torch.from_numpy(b.astype(np.float32)))
        print(f"stream_files {fname}: our attention vs the reference's, {snr:.1f} dB")
        assert snr >= 30.0, (fname, snr)
