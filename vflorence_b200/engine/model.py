"""An encoder-decoder model on the paged path.

Wraps a HuggingFace transformers BART-family model (``BartForConditionalGeneration``, or the
language model inside ``Florence2ForConditionalGeneration``). The encoder, the vision tower and
every projection run as stock torch modules on the GPU. The decoder is re-driven one token per
sequence: its self-attention goes through ``vflorence::self_attention`` (KV append + paged
decode) and its cross-attention through ``vflorence::cross_attention`` (paged encoder K/V), the
ops the reference's decoder calls (vflorence/models/bart.py:106-146). The q/k/v projections of
each decoder layer are fused into one GEMM and the encoder k/v projections into another, and the
kernels take the strided q/k/v views of the fused outputs directly. Each post-norm residual,
LayerNorm(h + sublayer(h)), and the embedding's LayerNorm(tokens + positions) run as one
launch of ``paged_ops.add_layernorm`` where it is built for the model's width and dtype. In
float32 steps of at most 16 rows every linear layer is one ``paged_ops.decode_linear`` launch.
"""

from __future__ import annotations

import contextlib
from types import SimpleNamespace

import torch
import torch.nn.functional as F
from transformers.activations import ACT2FN

from .. import paged_ops
from ..attention import decoder_cross_attention, decoder_self_attention


class _Layer:
    """One decoder layer's weights, plus the attribute slots PagedKVCache.bind fills."""

    def __init__(self, hf_layer):
        sa, ca = hf_layer.self_attn, hf_layer.encoder_attn
        cat = lambda *ms: torch.cat([m.weight for m in ms], 0)  # noqa: E731
        catb = lambda *ms: torch.cat([m.bias for m in ms], 0) if ms[0].bias is not None else None  # noqa: E731
        self.w_qkv, self.b_qkv = cat(sa.q_proj, sa.k_proj, sa.v_proj), catb(sa.q_proj, sa.k_proj, sa.v_proj)
        self.self_out = sa.out_proj
        self.ln_self = hf_layer.self_attn_layer_norm
        self.cross_q = ca.q_proj
        self.w_kv, self.b_kv = cat(ca.k_proj, ca.v_proj), catb(ca.k_proj, ca.v_proj)
        self.cross_out = ca.out_proj
        self.ln_cross = hf_layer.encoder_attn_layer_norm
        self.fc1, self.fc2 = hf_layer.fc1, hf_layer.fc2
        self.ln_final = hf_layer.final_layer_norm
        self.self_attn = SimpleNamespace(k_cache=None, v_cache=None)
        self.encoder_attn = SimpleNamespace(k_cache=None, v_cache=None)


class PagedSeq2Seq:
    def __init__(self, hf_model, fused_layernorm: bool = True, skinny_linear: bool = True):
        cfg = hf_model.config
        self.is_florence2 = cfg.model_type == "florence2"
        lm_cfg = cfg.get_text_config()
        self.hf = hf_model
        lm = hf_model.model.language_model if self.is_florence2 else hf_model.model
        self.lm = lm
        dec = lm.decoder
        self.embed_tokens = dec.embed_tokens
        self.pos_weight = dec.embed_positions.weight
        self.pos_offset = getattr(dec.embed_positions, "offset", 2)
        self.ln_embed = dec.layernorm_embedding
        self.layers = [_Layer(layer) for layer in dec.layers]
        self.num_heads = lm_cfg.decoder_attention_heads
        self.d_model = lm_cfg.d_model
        self.head_dim = self.d_model // self.num_heads
        self.scale = self.head_dim ** -0.5
        for L in self.layers:
            for attn in (L.self_attn, L.encoder_attn):
                attn.num_heads, attn.head_dim = self.num_heads, self.head_dim
        self.act = ACT2FN[lm_cfg.activation_function]
        self.lm_head = hf_model.lm_head
        self.final_logits_bias = getattr(hf_model, "final_logits_bias", None)
        self.vocab_size = self.lm_head.out_features
        # the vocabulary projection padded to a multiple of 64 rows: logit rows of an odd vocab
        # size (51289, 50265) are not 16-byte aligned, which keeps the GEMM off its fast kernels
        w, b = self.lm_head.weight, self.lm_head.bias
        pad = -self.vocab_size % 64
        if pad:
            w = torch.cat([w, w.new_zeros(pad, w.shape[1])])
            b = None if b is None else torch.cat([b, b.new_zeros(pad)])
        self.w_head, self.b_head = w, b
        self.dtype = self.pos_weight.dtype
        self.device = self.pos_weight.device
        self.image_token_id = getattr(cfg, "image_token_id", None)
        norms = [self.ln_embed] + [n for L in self.layers for n in (L.ln_self, L.ln_cross, L.ln_final)]
        self.fused_layernorm = (fused_layernorm and self.device.type == "cuda"
                                and all(isinstance(n, torch.nn.LayerNorm) and n.weight is not None
                                        and tuple(n.normalized_shape) == (self.d_model,) for n in norms)
                                and paged_ops.add_layernorm_supported(self.dtype, self.d_model))
        # float32 steps of at most 16 rows: the linear layers as weight-streaming launches
        # (paged_ops.decode_linear) instead of library GEMMs; fc1's activation fused when it is
        # the exact GELU
        self.skinny_linear = skinny_linear and self.device.type == "cuda" and self.dtype == torch.float32
        self.fuse_gelu = lm_cfg.activation_function == "gelu"

    # ------------------------------------------------------------------------------- encoder
    @torch.inference_mode()
    def encode(self, input_ids: torch.Tensor, pixel_values: torch.Tensor | None = None,
               attention_mask: torch.Tensor | None = None, phase=None) -> torch.Tensor:
        """Encoder hidden states [G, S, d_model] for a batch of prompts (right-padded and masked
        when their lengths differ; padded positions are never paged). ``phase(name)`` returns a
        context manager bracketing the vision tower and the text encoder (timing), if given."""
        phase = phase or (lambda name: contextlib.nullcontext())
        attention_mask = self._encoder_mask(attention_mask)
        if pixel_values is None:
            with phase("text_encoder"):
                return self.lm.encoder(input_ids=input_ids, attention_mask=attention_mask).last_hidden_state
        with phase("vision_tower"):
            feats = self.hf.model.get_image_features(pixel_values.to(self.dtype)).pooler_output
        with phase("text_encoder"):
            embeds = self.lm.get_input_embeddings()(input_ids)
            mask = (input_ids == self.image_token_id).unsqueeze(-1).expand_as(embeds)
            embeds = embeds.masked_scatter(mask, feats.to(embeds.dtype))
            return self.lm.encoder(inputs_embeds=embeds, attention_mask=attention_mask).last_hidden_state

    def _encoder_mask(self, mask: torch.Tensor | None):
        """The padding mask [G, S] as the prepared 4-D mask the encoder's attention takes (a 4-D
        mask is passed on as is), so that no host read of the mask stalls the stream: boolean
        (True = attend) for sdpa, additive for eager; other implementations get the 2-D mask."""
        if mask is None:
            return None
        impl = self.lm.config._attn_implementation
        g, s = mask.shape
        keep = mask.bool()[:, None, None, :].expand(g, 1, s, s)
        if impl == "sdpa":
            return keep
        if impl == "eager":
            add = torch.zeros(keep.shape, dtype=self.dtype, device=mask.device)
            return add.masked_fill(~keep, torch.finfo(self.dtype).min)
        return mask

    def cross_kv(self, layer: int, hidden: torch.Tensor):
        """Encoder K/V of one decoder layer as [G*S, H, head_dim] views of one fused GEMM."""
        L = self.layers[layer]
        kv = F.linear(hidden.reshape(-1, self.d_model), L.w_kv, L.b_kv)
        k, v = kv.chunk(2, dim=-1)
        shape = (kv.shape[0], self.num_heads, self.head_dim)
        return k.reshape(shape), v.reshape(shape)

    # ------------------------------------------------------------------------------- decoder
    def _linear(self, x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None, act: bool = False) -> torch.Tensor:
        """``x @ w.T + b`` (then the model's activation when ``act``): one decode_linear launch for a
        few float32 rows, else the library GEMM."""
        if self.skinny_linear and paged_ops.decode_linear_supported(x.dtype, x.shape[0], w.shape[0], w.shape[1]):
            if not act:
                return paged_ops.decode_linear(x, w, b)
            if self.fuse_gelu:
                return paged_ops.decode_linear(x, w, b, "gelu")
            return self.act(paged_ops.decode_linear(x, w, b))
        y = F.linear(x, w, b)
        return self.act(y) if act else y

    def _add_norm(self, h: torch.Tensor, x: torch.Tensor, norm: torch.nn.LayerNorm) -> torch.Tensor:
        """``norm(h + x)``: one fused launch, or the add and the module."""
        if self.fused_layernorm:
            return paged_ops.add_layernorm(h, x, norm.weight, norm.bias, norm.eps)
        return norm(h + x)

    @torch.inference_mode()
    def decode(self, input_ids: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
        """One decoder step: logits [B, vocab] for one new token per sequence. The per-step
        Context (slot mapping, block tables, cross staging) must be set."""
        B = input_ids.shape[0]
        h = self._add_norm(self.embed_tokens(input_ids), F.embedding(positions + self.pos_offset, self.pos_weight),
                           self.ln_embed)
        shape = (B, self.num_heads, self.head_dim)
        lin = self._linear
        for i, L in enumerate(self.layers):
            q, k, v = (t.reshape(shape) for t in lin(h, L.w_qkv, L.b_qkv).chunk(3, dim=-1))
            a = decoder_self_attention(q, k, v, L.self_attn.k_cache, L.self_attn.v_cache, self.scale)
            h = self._add_norm(h, lin(a.reshape(B, self.d_model), L.self_out.weight, L.self_out.bias), L.ln_self)
            c = decoder_cross_attention(lin(h, L.cross_q.weight, L.cross_q.bias).reshape(shape), i, self.scale)
            h = self._add_norm(h, lin(c.reshape(B, self.d_model), L.cross_out.weight, L.cross_out.bias), L.ln_cross)
            ff = lin(h, L.fc1.weight, L.fc1.bias, act=True)
            h = self._add_norm(h, lin(ff, L.fc2.weight, L.fc2.bias), L.ln_final)
        logits = lin(h, self.w_head, self.b_head)[:, : self.vocab_size]
        if self.final_logits_bias is not None:
            logits = logits + self.final_logits_bias
        return logits
