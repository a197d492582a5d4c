"""CPU oracle of the FP8 Einsum / GMLP contraction path.  TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may import
this package, and only as the checker or the timed CPU baseline; the product path
(macrogpt_jax_b200) never imports it.

What it restates (reference file:line, relative to the macrogpt-jax repository):
  * Einsum forward  `jnp.einsum(self.einsum_expr, x, self.w.value)`  ueaj/model/einsum.py:243,
    with the expression parsing of ueaj/model/einsum.py:81-147;
  * GMLP  `up, gate = fused_proj(x); gate = swish(gate); down(up * gate)`
    ueaj/model/mlp.py:78-115 (fused weight order [up, gate], ueaj/llama/weight_loader.py:131);
  * fp8 casts of custom_astype  ueaj/utils/gradutils.py:15-54, whose rounding is that of
    ml_dtypes 0.5.4 (requirements.txt:38);
  * the per-tensor current-scaling recipe (amax -> s = FMAX/amax -> RNE(x*s), fp32
    accumulate, bf16 out), which the reference does not contain: it is the recipe the
    FP8 mode is specified with, composed here from the primitives above;
  * RMSNorm.__call__  ueaj/model/rmsnorm.py:68-84 (norm.py), with the summation order and
    the rsqrt the CUDA kernel uses;
  * the next-token loss on the lm_head logits (xent.py): ntp_args / chunked_softmax_cross_entropy
    ueaj/opt/next_token_loss.py:13-174 and LlamaModel.get_logits ueaj/model/model.py:140-165;
  * Muon's Newton-Schulz orthogonalisation (muon.py): ueaj/opt/multiscale.py:110-200 and the
    optax 0.2.6 iteration it maps over the slices of a weight;
  * RoPE and the softmax attention of SoftmaxAttention (attention.py): ueaj/model/rope.py:10-104
    and the kvax flash_attention call of ueaj/model/soft_attn.py:186-196.

Parity pinning:
  * fp8 cast bytes: pinned.  fp8.py's own round-to-nearest-even cast is checked against
    ml_dtypes 0.5.4 (the reference's pinned cast library) on every bf16 bit pattern.
  * contraction / gating results: parity unpinned.  The reference's JAX program cannot run
    here (jax, flax, optax absent, no network) and the reference ships no golden vectors;
    these functions are restatements, checked against an independent einsum (torch) only.
"""
from . import attention, fp8, muon, norm, path, xent  # noqa: F401
