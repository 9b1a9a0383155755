"""DSL texts of the Llama-style decoders used by the benchmark configurations.

The graphs take precomputed token embeddings as input rows (as the
reference's models/llama3_style.tkm does) and end in a softmax cross-entropy
over the vocabulary; FC layers carry biases, as every FC does in the DSL.
"""


def llama_dsl(layers, d_model, q_heads, kv_heads, head_dim, ffn, vocab, seq, theta, loss=True):
    kv = kv_heads * head_dim
    head = f"  head: RMSNorm -> FC({vocab})" + (" -> SoftmaxCE" if loss else "")
    body = f"""attention: {{
  branch: RMSNorm -> {{
    q: FC({q_heads * head_dim}) -> RoPE(theta={theta})
    k: FC({kv}) -> RoPE(theta={theta})
    v: FC({kv})
  }} -> GQA(q={q_heads}, kv={kv_heads}, d={head_dim}, causal=true) -> FC({d_model})
  skip: Identity
}} -> Add
ffn: {{
  branch: RMSNorm -> {{
    gate: FC({ffn}) -> SiLU
    up: FC({ffn})
  }} -> Mul -> FC({d_model})
  skip: Identity
}} -> Add"""
    if layers > 1:
        # the DSL's loop macro repeats a block only for counts above one
        # (src/tkm_core.c:219-241); a single layer is written out
        flow = f"  layer x {layers}: {{\n" + _indent(body, 4) + "\n  }"
    else:
        flow = _indent(body, 2)
    return f"""input: 1x{seq}x{d_model}
prng: pcg32
flow:
{flow}
{head}
"""


def _indent(text, n):
    return "\n".join(" " * n + line for line in text.splitlines())


# Configuration 1: 2 layers, d_model 256, 4 heads x 64, SwiGLU 688, vocab 1024,
# batch 4 x seq 128 (tied embeddings are handled by the caller).
C1 = dict(layers=2, d_model=256, q_heads=4, kv_heads=4, head_dim=64, ffn=688, vocab=1024, seq=128, theta=10000,
          batch=4)

# Configuration 4: ~1B decoder, 16 layers, d_model 2048, GQA 32/8 x 64,
# SwiGLU 5632, vocab 32000, RoPE theta 500000, seq 2048, 8 sequences per GPU.
C4 = dict(layers=16, d_model=2048, q_heads=32, kv_heads=8, head_dim=64, ffn=5632, vocab=32000, seq=2048,
          theta=500000, batch=8)


def dsl_for(cfg, loss=True):
    keys = ("layers", "d_model", "q_heads", "kv_heads", "head_dim", "ffn", "vocab", "seq", "theta")
    return llama_dsl(*(cfg[k] for k in keys), loss=loss)
