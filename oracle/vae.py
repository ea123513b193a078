"""Oracle: the VAE bridge of the production drafter (fp32, CPU, test infrastructure).

Restates ``TransformerHiddenVAE.encode_sequence`` / ``decode_sequence`` (reference
``src/chain_flow/vae/transformer_hidden.py:51-67``: in-projection + learned positions, a stack of
pre-LN ``nn.TransformerEncoderLayer`` (bidirectional self-attention, GELU FFN of 4x width), a
final LayerNorm, then ``mu`` or the out-projection) and ``TreeVAEFlowDrafter.predict_hidden``
(``src/chain_flow/drafters/tree_vae_flow.py:163-175``: encode the context, integrate the flow
in latent space, decode). Weights use the reference's state-dict names under ``vae.``.
"""
from __future__ import annotations

import torch.nn.functional as F

from .flow import FlowConfig, integrate, layer_norm, mha


def encoder_layer(x, W, prefix: str, heads: int):
    """nn.TransformerEncoderLayer(norm_first=True, activation='gelu'), no mask."""
    a = layer_norm(x, W[prefix + "norm1.weight"], W[prefix + "norm1.bias"])
    x = x + mha(a, a, W, prefix + "self_attn.", heads, None)
    f = layer_norm(x, W[prefix + "norm2.weight"], W[prefix + "norm2.bias"])
    u = F.gelu(f @ W[prefix + "linear1.weight"].T + W[prefix + "linear1.bias"])
    return x + u @ W[prefix + "linear2.weight"].T + W[prefix + "linear2.bias"]


def _stack(W, x, side: str, layers: int, heads: int):
    for i in range(layers):
        x = encoder_layer(x, W, f"vae.{side}.layers.{i}.", heads)
    return layer_norm(x, W[f"vae.{side}_norm.weight"], W[f"vae.{side}_norm.bias"])


def vae_encode(W, hidden, layers: int, heads: int):
    """[B, L, H] -> mu [B, L, latent] (transformer_hidden.py:51-58)."""
    L = hidden.shape[1]
    x = hidden @ W["vae.encoder_in.weight"].T + W["vae.encoder_in.bias"] + W["vae.encoder_pos.weight"][:L]
    x = _stack(W, x, "encoder", layers, heads)
    return x @ W["vae.mu.weight"].T + W["vae.mu.bias"]


def vae_decode(W, z, layers: int, heads: int):
    """[B, L, latent] -> [B, L, H] (transformer_hidden.py:60-67)."""
    L = z.shape[1]
    x = z @ W["vae.decoder_in.weight"].T + W["vae.decoder_in.bias"] + W["vae.decoder_pos.weight"][:L]
    x = _stack(W, x, "decoder", layers, heads)
    return x @ W["vae.decoder_out.weight"].T + W["vae.decoder_out.bias"]


def predict_hidden_vae(W, cfg: FlowConfig, vae_layers: int, vae_heads: int, ctx, z0):
    """decode(integrate(encode(ctx), z0)); cfg describes the latent-space flow."""
    return vae_decode(W, integrate(W, cfg, vae_encode(W, ctx, vae_layers, vae_heads), z0), vae_layers, vae_heads)
