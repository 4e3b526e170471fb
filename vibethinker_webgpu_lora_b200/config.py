"""Model configuration (src/config.js:27-48 of the reference)."""

QWEN25_3B = {
    "hiddenSize": 2048,
    "numLayers": 36,
    "numHeads": 16,
    "numKVHeads": 2,
    "headDim": 128,
    "intermediateSize": 11008,
    "vocabSize": 151936,
    "rmsNormEps": 1e-6,
    "ropeTheta": 1000000.0,
    "tieWordEmbeddings": True,
    "attentionBias": True,
}


def small_config(layers: int = 2, vocab: int = 4096, inter: int = 1024) -> dict:
    """Reduced-depth/width variant with the same head geometry (16 Q / 2 KV
    heads of 128), used for fast parity tests."""
    c = dict(QWEN25_3B)
    c.update(numLayers=layers, vocabSize=vocab, intermediateSize=inter)
    return c
