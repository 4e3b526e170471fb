"""Whole-prompt prefill on the tensor cores (prefillTc, the default) against
the oracle's restatement of prefillBatch (runtime.js:1936-2087): logits and
hidden state after the prompt, the K/V cache it leaves (decoding continues
from it), _prefillFull and _prefillChunked, f32 and f16 staging, LoRA.

Bars: the f32 path within the north-star bars (max-abs 1e-2, mean-rel 1e-3)
with the measured distance printed; the f16 path (RMSNORM_T_F16, ROPE_T_F16,
SILUMUL_F16 roundings) amplifies f32-level differences into whole f16 ulps,
and is held to the same bars on these 2-3 layer models."""
import numpy as np
import pytest

from oracle import oracle as O
import vibethinker_webgpu_lora_b200 as E
from vibethinker_webgpu_lora_b200.config import small_config

pytestmark = pytest.mark.gpu
SEED = 0xE6B00000
TIE_BOUND = 2e-3


def dist(got, ref):
    d = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    return d.max(), d.mean() / max(np.abs(ref.astype(np.float64)).mean(), 1e-12)


def close(got, ref, max_abs=1e-2, mean_rel=1e-3):
    m, r = dist(got, ref)
    assert m <= max_abs and r <= mean_rel, f"max abs {m:.3g} mean rel {r:.3g}"


@pytest.mark.parametrize("f16", [False, True])
@pytest.mark.parametrize("T,chunk", [(150, 0), (300, 128), (33, 0), (1, 0), (64, 32)])
def test_prefill_tc_vs_oracle(cuda, f16, T, chunk):
    cfg = small_config(layers=3, vocab=5000, inter=1024)
    rt = E.QwenB200(cfg, dict(maxCtx=512, useF16=f16, prefillChunkSize=chunk)).build("synthetic", seed=SEED)
    orc = O.OracleModel(cfg, 512, f16, SEED)
    prompt = O.token_ids(T, 0xE6B00020 + T, cfg["vocabSize"])
    ref = orc.prefill(prompt, chunk)
    rt.prefillBatch(prompt)
    got = rt.readLogits()
    print(f"prefill T={T} chunk={chunk} f16={f16}: logits {dist(got, ref)} hidden "
          f"{dist(rt.readHidden(), orc.hidden())}")
    close(got, ref)
    close(rt.readHidden(), orc.hidden())
    # decoding continues from the cache the pass left
    first = rt.argmaxLogits()
    ids = rt.decodeBatch(T, 8)
    want, margins = [], []
    logits = ref
    for g in range(9):
        s = np.sort(logits.astype(np.float64))
        want.append(O.argmax(logits))
        margins.append(s[-1] - s[-2])
        if g < 8:
            logits = orc.step(want[-1], T + g)
    for i, (a, b) in enumerate(zip([first] + ids, want)):
        if a != b:
            assert margins[i] < TIE_BOUND, f"token {i}: {a} != {b}, margin {margins[i]:.3g}"
            break


def test_prefill_tc_lora(cuda):
    """loraBatchDelta (runtime.js:1814-1843) on every projection of the
    pass: the adapter's prefill logits meet the oracle's."""
    cfg = small_config(layers=2, vocab=3000)
    prompt = O.token_ids(70, 0xE6B00031, cfg["vocabSize"])
    rt = E.QwenB200(cfg, dict(maxCtx=128)).build("synthetic", seed=SEED)
    a = E.synthetic_adapter(rt, 0xA1, rank=8, alpha=16)
    rt.setLora(a)
    rt.prefillBatch(prompt)
    orc = O.OracleModel(cfg, 128, True, SEED)
    orc.lora_synth(0xA1, 8, 2.0)
    ref = orc.prefill(prompt)
    got = rt.readLogits()
    print("prefill lora:", dist(got, ref))
    close(got, ref)
    rt.clearLora()
    rt.prefillBatch(prompt)
    base = O.OracleModel(cfg, 128, True, SEED).prefill(prompt)
    close(rt.readLogits(), base)
    a.destroy()


def test_prefill_tc_repeatable_and_prefill_after_decode(cuda):
    """Two prefills of the same prompt give the same bits; a prefill after
    decoding restarts the stream at position 0."""
    cfg = small_config(layers=2, vocab=3000)
    prompt = O.token_ids(90, 0xE6B00032, cfg["vocabSize"])
    rt = E.QwenB200(cfg, dict(maxCtx=256)).build("synthetic", seed=SEED)
    rt.prefillBatch(prompt)
    a = rt.readLogits()
    rt.decodeBatch(90, 5)
    rt.prefillBatch(prompt)
    assert np.array_equal(a, rt.readLogits())


@pytest.mark.slow
@pytest.mark.parametrize("f16", [False, True])
def test_full_model_prefill_tc(cuda, f16):
    """Qwen2.5-3B shape, 32-token prompt: logits after prefillBatch against
    the oracle's prefillBatch (36 layers; the f16 path's bar is its measured
    f16 distance, printed)."""
    cfg = E.QWEN25_3B
    prompt = O.token_ids(32, 0xE6B00010, cfg["vocabSize"])
    orc = O.OracleModel(cfg, 64, f16, SEED)
    ref = orc.prefill(prompt)
    rt = E.QwenB200(cfg, dict(maxCtx=64, useF16=f16)).build("synthetic", seed=SEED)
    rt.prefillBatch(prompt)
    got = rt.readLogits()
    m, r = dist(got, ref)
    print(f"full-model prefill f16={f16}: max abs {m:.3g} mean rel {r:.3g}")
    if not f16:
        close(got, ref)
    else:
        close(got, ref, 3e-2, 5e-3)
    s = np.sort(ref.astype(np.float64))
    assert rt.argmaxLogits() == O.argmax(ref) or s[-1] - s[-2] < TIE_BOUND
