"""Random-init Transformers backbones with given weights: the Qwen3_5Model (full-attention and Gated DeltaNet layers)
and Gemma4TextModel (5 sliding : 1 global layers) that the reference's ``families.*.Packed`` wrap, built from the
seeded weights of ``karpo_decision_b200.synthetic``. Used by the golden generator (tests/golden/make_golden.py) to run
the reference, and by the drop-in tests to build ``Packed.from_backbone`` from the same modules. Needs only
Transformers, not the reference."""

from __future__ import annotations

import numpy as np
import torch

from karpo_decision_b200.synthetic import Spec


def to_torch(weights: dict[str, np.ndarray], key: str) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(weights[key]))


def qwen_backbone(spec: Spec, weights: dict[str, np.ndarray]):
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5Config
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5Model

    rot = int(spec.head_dim * spec.partial_rotary)
    half = rot // 2
    section = list(spec.mrope_section) if spec.mrope_section else [half - 2 * (half // 3), half // 3, half // 3]
    text = dict(vocab_size=spec.vocab, hidden_size=spec.hidden, intermediate_size=spec.intermediate,
                num_hidden_layers=spec.layers, num_attention_heads=spec.heads, num_key_value_heads=spec.kv_heads,
                head_dim=spec.head_dim, rms_norm_eps=spec.eps, layer_types=spec.layer_types(),
                rope_parameters={"rope_type": "default", "rope_theta": spec.rope_theta,
                                 "partial_rotary_factor": spec.partial_rotary, "mrope_section": section},
                attention_bias=False, hidden_act="silu", linear_num_key_heads=spec.lin_k_heads,
                linear_num_value_heads=spec.lin_v_heads, linear_key_head_dim=spec.lin_k_dim,
                linear_value_head_dim=spec.lin_v_dim, linear_conv_kernel_dim=spec.conv_kernel)
    config = Qwen3_5Config(text_config=text, vision_config={"depth": 1, "hidden_size": 32, "intermediate_size": 64,
                                                           "num_heads": 2, "out_hidden_size": spec.hidden},
                           image_token_id=spec.vocab - 1)  # the fixtures' image token (the last id)
    config._attn_implementation = "sdpa"
    model = Qwen3_5Model(config).float().eval()
    lm = model.language_model
    with torch.no_grad():
        lm.embed_tokens.weight.copy_(to_torch(weights, "embed_tokens"))
        lm.norm.weight.copy_(to_torch(weights, "norm"))
        for i, layer in enumerate(lm.layers):
            p = f"layers.{i}."
            layer.block_type = layer.layer_type  # harness alias (Transformers 5.5 naming)
            if layer.layer_type == "linear_attention":
                la = layer.linear_attn
                for name in ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a", "out_proj"):
                    getattr(la, name).weight.copy_(to_torch(weights, p + "linear_attn." + name))
                la.conv1d.weight.copy_(to_torch(weights, p + "linear_attn.conv1d")[:, None, :])
                la.A_log.copy_(to_torch(weights, p + "linear_attn.A_log"))
                la.dt_bias.copy_(to_torch(weights, p + "linear_attn.dt_bias"))
                la.norm.weight.copy_(to_torch(weights, p + "linear_attn.norm"))
            else:
                a = layer.self_attn
                for name in ("q_proj", "k_proj", "v_proj", "o_proj"):
                    getattr(a, name).weight.copy_(to_torch(weights, p + name))
                a.q_norm.weight.copy_(to_torch(weights, p + "q_norm"))
                a.k_norm.weight.copy_(to_torch(weights, p + "k_norm"))
            for name in ("gate_proj", "up_proj", "down_proj"):
                getattr(layer.mlp, name).weight.copy_(to_torch(weights, p + name))
            layer.input_layernorm.weight.copy_(to_torch(weights, p + "input_layernorm"))
            layer.post_attention_layernorm.weight.copy_(to_torch(weights, p + "post_attention_layernorm"))
    return model


def gemma_lm(spec: Spec, weights: dict[str, np.ndarray]):
    from transformers.models.gemma4.configuration_gemma4 import Gemma4TextConfig
    from transformers.models.gemma4.modeling_gemma4 import Gemma4TextModel

    global_rope = {"rope_type": "default", "rope_theta": spec.rope_theta}
    if spec.global_rope == "proportional":
        global_rope = {"rope_type": "proportional", "rope_theta": spec.rope_theta,
                       "partial_rotary_factor": spec.global_partial_rotary}
    config = Gemma4TextConfig(
        vocab_size=spec.vocab, hidden_size=spec.hidden, intermediate_size=spec.intermediate,
        num_hidden_layers=spec.layers, num_attention_heads=spec.heads, num_key_value_heads=spec.kv_heads,
        head_dim=spec.head_dim, global_head_dim=spec.global_head_dim or spec.head_dim,
        num_global_key_value_heads=spec.global_kv_heads or spec.kv_heads, attention_k_eq_v=spec.k_eq_v,
        sliding_window=spec.window, layer_types=spec.layer_types(),
        hidden_size_per_layer_input=0, final_logit_softcapping=spec.logit_cap, rms_norm_eps=spec.eps,
        hidden_activation="gelu_pytorch_tanh",
        rope_parameters={"sliding_attention": {"rope_type": "default", "rope_theta": spec.rope_theta_local},
                         "full_attention": global_rope})
    config._attn_implementation = "sdpa"
    lm = Gemma4TextModel(config).float().eval()
    with torch.no_grad():
        lm.embed_tokens.weight.copy_(to_torch(weights, "embed_tokens"))
        lm.norm.weight.copy_(to_torch(weights, "norm"))
        for i, layer in enumerate(lm.layers):
            p = f"layers.{i}."
            a = layer.self_attn
            for name in ("q_proj", "k_proj", "v_proj", "o_proj"):
                if getattr(a, name) is not None:  # attention_k_eq_v global layers have no v_proj
                    getattr(a, name).weight.copy_(to_torch(weights, p + name))
            a.q_norm.weight.copy_(to_torch(weights, p + "q_norm"))
            a.k_norm.weight.copy_(to_torch(weights, p + "k_norm"))
            for name in ("gate_proj", "up_proj", "down_proj"):
                getattr(layer.mlp, name).weight.copy_(to_torch(weights, p + name))
            for name in ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                         "post_feedforward_layernorm"):
                getattr(layer, name).weight.copy_(to_torch(weights, p + name))
            layer.layer_scalar.copy_(to_torch(weights, p + "layer_scalar"))
    return lm


def to_dtype(model: torch.nn.Module, dtype: torch.dtype) -> torch.nn.Module:
    """``model`` cast to ``dtype`` the way a checkpoint loaded in that dtype is: parameters and buffers cast, but the
    rotary embeddings' inverse frequencies kept in float32 (Transformers computes them in float32 at construction; a
    bf16 copy would put the rotation angles at long positions off by radians)."""
    kept = {name: buf.clone() for name, buf in model.named_buffers() if name.endswith("inv_freq")}
    model = model.to(dtype)
    for name, buf in kept.items():
        owner, _, attr = name.rpartition(".")
        module = model.get_submodule(owner) if owner else model
        setattr(module, attr, buf) if attr not in module._buffers else module._buffers.__setitem__(attr, buf)
    return model


