"""Host mirrors of the reference's window models, wired to the CUDA attention.

`GT_SW` mirrors `NeutronGT/models/gt_dist_node_level_single_window.py:505-680` and `Graphormer`
mirrors `NeutronGT/models/graphormer_dist_node_level.py:240-381`: same constructor arguments,
same submodule and parameter names (so a state_dict saved by the reference loads here
unchanged), same forward signature and return tuple
`(log_softmax(out), score_agg, [per-layer node scores], kv_cache)`.  The attention itself
is `attention.CoreAttention` (sparse: `csrc/spattn.cu`).  LayerNorm and Linear are
`layers.LayerNorm` / `layers.Linear`: the torch modules' parameters and math, with the LayerNorm
passes and the bias gradients on `csrc/rowops.cu`.

Behaviour kept from the reference on purpose (it changes results, so parity needs it):
* GT_SW's encoder feeds the FFN with the attention branch `y`, not the residual stream
  (`…single_window.py:345`), ignores `ffn_dim` (FFN width is 2*hidden, :322-323), and never
  applies `self_attention_norm` (:311);
* Graphormer is pre-LayerNorm with a GELU FFN of width `ffn_dim` and an output projection
  after attention (`graphormer…:139, 176-206`);
* parameters are drawn by `init_params` (`…single_window.py:22-28`): Linear N(0, 0.02/sqrt(L)),
  bias 0, Embedding N(0, 0.02).
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from .attention import CoreAttention
from .layers import LayerNorm, Linear


def init_params(module, n_layers):
    if isinstance(module, nn.Linear):
        module.weight.data.normal_(mean=0.0, std=0.02 / math.sqrt(n_layers))
        if module.bias is not None:
            module.bias.data.zero_()
    if isinstance(module, nn.Embedding):
        module.weight.data.normal_(mean=0.0, std=0.02)


class CentralityEncodingLayer(nn.Module):
    """Degree embeddings.  Graphormer clamps degrees before the lookup (`graphormer…:217-220`);
    GT_SW clamps after it, which leaves the lookup unclamped (`…single_window.py:398-405`)."""

    def __init__(self, hidden_dim, num_in_degree=512, num_out_degree=512, clamp_first=False):
        super().__init__()
        self.num_in_degree = num_in_degree
        self.num_out_degree = num_out_degree
        self.clamp_first = clamp_first
        self.in_degree_encoder = nn.Embedding(num_in_degree + 1, hidden_dim, padding_idx=0)
        self.out_degree_encoder = nn.Embedding(num_out_degree + 1, hidden_dim, padding_idx=0)

    def forward(self, x, in_degree, out_degree):
        if self.clamp_first:
            in_degree = in_degree.clamp(max=self.num_in_degree - 1)
            out_degree = out_degree.clamp(max=self.num_out_degree - 1)
        return x + self.in_degree_encoder(in_degree.long()) + self.out_degree_encoder(out_degree.long())


class AttnBias(nn.Module):
    """Spatial-position bias [b, H, s, s] (`…single_window.py:413-497`; edge bias is disabled there)."""

    def __init__(self, num_heads, num_spatial=512, num_edges=1024, max_dist=32, edge_dim=32):
        super().__init__()
        self.num_heads = num_heads
        self.max_dist = max_dist
        self.edge_dim = edge_dim
        self.spatial_pos_encoder = nn.Embedding(num_spatial, num_heads, padding_idx=0)
        self.edge_feature_encoder = nn.Embedding(num_edges + 1, edge_dim, padding_idx=0)
        self.edge_pos_encoder = nn.Embedding(max_dist, edge_dim * num_heads)

    def forward(self, spatial_pos, edge_input):
        return self.spatial_pos_encoder(spatial_pos.long()).permute(0, 3, 1, 2)


class _DistributedAttentionSlot(nn.Module):
    """Keeps the reference's `dist_attn` submodule (it wraps `local_attn`; no parameters)."""

    def __init__(self, local_attention):
        super().__init__()
        self.local_attn = local_attention


def _kv_with_cache(mha, x, batch_size, dup_nodes_kv_cache, layer):
    """K/V with the duplicate-node cache splice of `…single_window.py:264-283`."""
    if dup_nodes_kv_cache is None:
        k = mha.linear_k(x).view(batch_size, -1, mha.num_heads, mha.att_size)
        v = mha.linear_v(x).view(batch_size, -1, mha.num_heads, mha.att_size)
        return k, v, k, v
    k_cache, v_cache = dup_nodes_kv_cache[layer]
    n_dup = k_cache.size(0)
    assert n_dup <= x.shape[1], f"Cache size {n_dup} > input seq_len {x.shape[1]}"
    x_dyn = x[:, n_dup:, :]
    k_dyn = mha.linear_k(x_dyn).view(batch_size, -1, mha.num_heads, mha.att_size)
    v_dyn = mha.linear_v(x_dyn).view(batch_size, -1, mha.num_heads, mha.att_size)
    k = torch.cat([k_cache.unsqueeze(0).expand(batch_size, -1, -1, -1), k_dyn], dim=1)
    v = torch.cat([v_cache.unsqueeze(0).expand(batch_size, -1, -1, -1), v_dyn], dim=1)
    return k, v, k, v


class MultiHeadAttention(nn.Module):
    """`…single_window.py:230-302` (GT) / `graphormer…:130-173` (with `output_layer`)."""

    def __init__(self, hidden_size, attention_dropout_rate, num_heads, output_layer=False):
        super().__init__()
        self.num_heads = num_heads
        self.att_size = hidden_size // num_heads
        self.linear_q = Linear(hidden_size, num_heads * self.att_size)
        self.linear_k = Linear(hidden_size, num_heads * self.att_size)
        self.linear_v = Linear(hidden_size, num_heads * self.att_size)
        self.local_attn = CoreAttention(hidden_size, attention_dropout_rate, num_heads)
        if output_layer:
            self.output_layer = Linear(num_heads * self.att_size, hidden_size)
        else:
            self.dist_attn = _DistributedAttentionSlot(self.local_attn)
            self.output_layer = None

    def forward(self, x, attn_bias=None, edge_index=None, attn_type=None, mask=None, pruning_mask=None,
                dup_nodes_kv_cache=None, layer: int = 0):
        orig = x.size()
        b = x.size(0)
        q = self.linear_q(x).view(b, -1, self.num_heads, self.att_size)
        k, v, ck, cv = _kv_with_cache(self, x, b, dup_nodes_kv_cache, layer)
        x, score = self.local_attn(q, k, v, attn_bias, edge_index, attn_type, mask=mask, pruning_mask=pruning_mask)
        if self.output_layer is not None:
            x = self.output_layer(x)
        assert x.size() == orig
        return x, score, [ck, cv]


class GTEncoderLayer(nn.Module):
    def __init__(self, hidden_size, ffn_size, dropout_rate, attention_dropout_rate, num_heads):
        super().__init__()
        self.self_attention_norm = LayerNorm(hidden_size)
        self.self_attention = MultiHeadAttention(hidden_size, attention_dropout_rate, num_heads)
        self.self_attention_dropout = nn.Dropout(dropout_rate)
        self.O = Linear(hidden_size, hidden_size)
        self.layer_norm1 = LayerNorm(hidden_size)
        self.FFN_layer1 = Linear(hidden_size, hidden_size * 2)
        self.FFN_layer2 = Linear(hidden_size * 2, hidden_size)
        self.layer_norm2 = LayerNorm(hidden_size)

    def forward(self, x, attn_bias=None, edge_index=None, attn_type=None, mask=None, pruning_mask=None,
                dup_nodes_kv_cache=None, layer: int = 0):
        y, score, cache = self.self_attention(x, attn_bias, edge_index=edge_index, attn_type=attn_type,
                                              pruning_mask=pruning_mask, mask=mask,
                                              dup_nodes_kv_cache=dup_nodes_kv_cache, layer=layer)
        y = self.O(self.self_attention_dropout(y))
        x = self.layer_norm1(x + y)
        y = self.FFN_layer2(self.self_attention_dropout(F.relu(self.FFN_layer1(y))))
        x = self.layer_norm2(x + y)
        return x, score, cache


class MLPReadout(nn.Module):
    def __init__(self, input_dim, output_dim, L=2):
        super().__init__()
        layers = [Linear(input_dim // 2 ** l, input_dim // 2 ** (l + 1), bias=True) for l in range(L)]
        layers.append(Linear(input_dim // 2 ** L, output_dim, bias=True))
        self.FC_layers = nn.ModuleList(layers)
        self.L = L

    def forward(self, x):
        for l in range(self.L):
            x = F.relu(self.FC_layers[l](x))
        return self.FC_layers[self.L](x)


def _collect_cache(dup_nodes_kv_cache, layer_caches):
    """The reference's cache bookkeeping (`…single_window.py:629-678`): only layers that ran
    with a cache contribute, so a None cache stays None."""
    new = []
    for ck, cv in layer_caches:
        n_dup = 0
        if dup_nodes_kv_cache is not None and isinstance(dup_nodes_kv_cache, tuple) and len(dup_nodes_kv_cache) == 2:
            if dup_nodes_kv_cache[0] is not None:
                n_dup = dup_nodes_kv_cache[0].shape[0]
        if ck is not None and cv is not None and dup_nodes_kv_cache is not None and n_dup > 0:
            new.append((ck[:, :n_dup].squeeze(0).detach(), cv[:, :n_dup].squeeze(0).detach()))
        else:
            new.append((None, None))
    updated = dup_nodes_kv_cache
    if new and any(k is not None for k, _ in new):
        if updated is None:
            updated = [(k, v) if k is not None and v is not None else (None, None) for k, v in new]
        elif isinstance(updated, list):
            for i, (k, v) in enumerate(new):
                if k is not None and v is not None and i < len(updated):
                    updated[i] = (k, v)
    return updated


class GT_SW(nn.Module):
    def __init__(self, n_layers, num_heads, input_dim, hidden_dim, output_dim, attn_bias_dim, dropout_rate,
                 input_dropout_rate, attention_dropout_rate, ffn_dim, num_global_node, args, num_in_degree: int,
                 num_out_degree: int, num_spatial, num_edges, max_dist, edge_dim):
        super().__init__()
        self.args = args
        self.node_encoder = Linear(input_dim, hidden_dim)
        self.centrality_encoding = CentralityEncodingLayer(hidden_dim, num_in_degree, num_out_degree)
        self.attention_bias = AttnBias(num_heads, num_spatial, num_edges, max_dist, edge_dim)
        self.input_dropout = nn.Dropout(input_dropout_rate)
        self.layers = nn.ModuleList([GTEncoderLayer(hidden_dim, ffn_dim, dropout_rate, attention_dropout_rate, num_heads)
                                     for _ in range(n_layers)])
        self.MLP_layer = MLPReadout(hidden_dim, output_dim)
        self.downstream_out_proj = Linear(hidden_dim, output_dim)
        self.apply(lambda m: init_params(m, n_layers=n_layers))

    def forward(self, x, attn_bias, edge_index, in_degree, out_degree, spatial_pos, edge_input, perturb=None,
                attn_type=None, mask=None, pruning_mask=None, dup_nodes_kv_cache=None, part_id=None):
        x = x.unsqueeze(0)
        h = self.node_encoder(x)
        if getattr(self.args, "struct_enc", "False") == "True":
            h = self.centrality_encoding(h, in_degree.unsqueeze(0), out_degree.unsqueeze(0))
            bias = self.attention_bias(spatial_pos.unsqueeze(0), None)
            attn_bias = bias + attn_bias if attn_bias is not None else bias
        out = self.input_dropout(h)
        scores, caches = [], []
        for i, layer in enumerate(self.layers):
            out, score, cache = layer(out, attn_bias=attn_bias, edge_index=edge_index, attn_type=attn_type, mask=mask,
                                      dup_nodes_kv_cache=dup_nodes_kv_cache, layer=i)
            scores.append(score.detach())
            caches.append(cache)
        out = self.MLP_layer(out[0])
        return F.log_softmax(out, dim=1), None, scores, _collect_cache(dup_nodes_kv_cache, caches)


class GraphormerEncoderLayer(nn.Module):
    def __init__(self, hidden_size, ffn_size, dropout_rate, attention_dropout_rate, num_heads):
        super().__init__()
        self.self_attention_norm = LayerNorm(hidden_size)
        self.self_attention = MultiHeadAttention(hidden_size, attention_dropout_rate, num_heads, output_layer=True)
        self.self_attention_dropout = nn.Dropout(dropout_rate)
        self.ffn_norm = LayerNorm(hidden_size)
        self.ffn = nn.Module()
        self.ffn.layer1 = Linear(hidden_size, ffn_size)
        self.ffn.gelu = nn.GELU()
        self.ffn.layer2 = Linear(ffn_size, hidden_size)
        self.ffn_dropout = nn.Dropout(dropout_rate)

    def forward(self, x, attn_bias=None, edge_index=None, attn_type=None, mask=None, pruning_mask=None,
                dup_nodes_kv_cache=None, layer: int = 0):
        y = self.self_attention_norm(x)
        y, score, cache = self.self_attention(y, attn_bias, edge_index, attn_type=attn_type, mask=mask,
                                              pruning_mask=pruning_mask, dup_nodes_kv_cache=dup_nodes_kv_cache,
                                              layer=layer)
        x = x + self.self_attention_dropout(y)
        y = self.ffn.layer2(self.ffn.gelu(self.ffn.layer1(self.ffn_norm(x))))
        x = x + self.ffn_dropout(y)
        return x, score, cache


class Graphormer(nn.Module):
    def __init__(self, n_layers, num_heads, input_dim, hidden_dim, output_dim, attn_bias_dim, dropout_rate,
                 input_dropout_rate, attention_dropout_rate, ffn_dim, num_global_node, args, num_in_degree,
                 num_out_degree, num_spatial, num_edges, max_dist, edge_dim):
        super().__init__()
        self.args = args
        self.num_heads = num_heads
        self.node_encoder = Linear(input_dim, hidden_dim)
        self.centrality_encoding = CentralityEncodingLayer(hidden_dim, num_in_degree, num_out_degree, clamp_first=True)
        self.attention_bias = AttnBias(num_heads, num_spatial, num_edges, max_dist, edge_dim)
        self.input_dropout = nn.Dropout(input_dropout_rate)
        self.layers = nn.ModuleList([GraphormerEncoderLayer(hidden_dim, ffn_dim, dropout_rate, attention_dropout_rate,
                                                            num_heads) for _ in range(n_layers)])
        self.final_ln = LayerNorm(hidden_dim)
        self.downstream_out_proj = Linear(hidden_dim, output_dim)
        self.n_layers = n_layers
        self.apply(lambda m: init_params(m, n_layers=n_layers))

    def forward(self, x, attn_bias, edge_index, in_degree, out_degree, spatial_pos, edge_input, perturb=None,
                attn_type=None, mask=None, pruning_mask=None, dup_nodes_kv_cache=None, part_id=None):
        x = x.unsqueeze(0)
        h = self.node_encoder(x)
        if perturb is not None:
            h = h + perturb
        if getattr(self.args, "struct_enc", "False") == "True":
            h = self.centrality_encoding(h, in_degree.unsqueeze(0), out_degree.unsqueeze(0))
            bias = self.attention_bias(spatial_pos.unsqueeze(0), None)
            attn_bias = bias + attn_bias if attn_bias is not None else bias
        out = self.input_dropout(h)
        scores, caches = [], []
        for i, layer in enumerate(self.layers):
            out, score, cache = layer(out, attn_bias=attn_bias, edge_index=edge_index, attn_type=attn_type, mask=mask,
                                      pruning_mask=pruning_mask, dup_nodes_kv_cache=dup_nodes_kv_cache, layer=i)
            scores.append(score.detach() if score is not None else None)
            caches.append(cache)
        out = self.downstream_out_proj(self.final_ln(out)[0])
        return F.log_softmax(out, dim=1), None, scores, _collect_cache(dup_nodes_kv_cache, caches)
