"""CPU checks of the Qwen3-Next stack oracle (no GPU)."""
import numpy as np

from oracle import qwen_next as OQ


def _tiny():
    # the shapes of vates_b200.qwen_next.tiny_config, without importing torch code
    return OQ.Config(hidden=1024, vocab=2048, layers=4, full_attention_interval=4, q_heads=4,
                     kv_heads=1, head_dim=256, rope_dims=64, rope_base=10_000_000.0, eps=1e-6,
                     k_heads=2, v_heads=4, head_k=128, head_v=128, experts=16, top_k=4,
                     inter=128, group=64, bits=4, dense_scale=(0.001, 0.01),
                     dense_bias_mul=-7.5, expert_bias_mul=-7.5, unit_norms=False)


def test_accept_prefix():
    assert OQ.accept_prefix([1, 2, 3], [1, 2, 4]) == 2
    assert OQ.accept_prefix([1, 2, 3], [0, 2, 3]) == 0
    assert OQ.accept_prefix([5, 6], [5, 6, 7]) == 2


def test_spec_equals_greedy():
    """Speculative decoding with exact verify and direct commit emits the
    plain greedy tokens (the reference's lossless property, generate.py:
    338-352, 818-853), for both verify lengths."""
    m = OQ.Model(_tiny(), seed=4)
    prompt = np.random.default_rng(0).integers(0, 2048, 9).tolist()
    m.reset()
    logits = None
    for s in range(0, len(prompt), 4):
        logits, _ = m.forward(prompt[s:s + 4])
    greedy = [OQ.argmax(logits[-1])]
    while len(greedy) < 6:
        logits, _ = m.forward([greedy[-1]])
        greedy.append(OQ.argmax(logits[-1]))
    for V in (3, 4):
        toks, steps = OQ.spec_generate(m, prompt, 6, K=3, V=V)
        assert toks == greedy, (V, toks, greedy)


def test_rope_rotates_pairs():
    x = np.zeros((1, 2, 256), np.float32)
    x[0, :, 0] = 1.0
    y = OQ.rope(x, 3, 64, 10000.0)
    # position 3 and 4, dim 0 pairs with dim 32 at frequency 1
    assert np.allclose(y[0, 0, 0], np.cos(3.0), atol=1e-2)
    assert np.allclose(y[0, 0, 32], np.sin(3.0), atol=1e-2)
    assert np.allclose(y[0, 1, 32], np.sin(4.0), atol=1e-2)
    assert np.all(y[0, :, 64:] == 0)
