"""The model-forward call sites of the fused ops (svllm_ops.Model, DecodeGraphs).

Oracle: Hugging Face's Qwen3ForCausalLM and LlamaForCausalLM (llama3 rope scaling) with the same
random weights, run in bf16 on the same device, each request recomputed from its full token
sequence. Our forward runs the fused ops (embedding, add_rms_norm, qk_norm_rope_cache /
rope_cache, silu_and_mul, argmax) around torch GEMMs and a LibTorch attention over the paged KV
cache, so logits agree to bf16 rounding noise through two layers, not bit for bit: the bar is
max |logit difference| <= 2% of max |logit|, and the greedy tokens equal Hugging Face's argmax
wherever its top two logits differ by more than that bar.

Decode graphs are checked bit for bit against the eager decode at the same padded batch.
"""

from __future__ import annotations

import pytest
import torch

import svllm_ops

transformers = pytest.importorskip("transformers")

VOCAB, HIDDEN, INTER, LAYERS, HEADS, KV_HEADS, HEAD_DIM = 1000, 256, 512, 2, 4, 2, 64
BLOCK = 16
REL_BAR = 0.02


def tiny(arch: str, device: torch.device):
    """A two-layer random-weight model of `arch` and our Model over the same weights."""
    torch.manual_seed(0)
    common = dict(vocab_size=VOCAB, hidden_size=HIDDEN, intermediate_size=INTER,
                  num_hidden_layers=LAYERS, num_attention_heads=HEADS,
                  num_key_value_heads=KV_HEADS, head_dim=HEAD_DIM, tie_word_embeddings=True,
                  max_position_embeddings=4096)
    if arch == "qwen3":
        hf_cfg = transformers.Qwen3Config(rms_norm_eps=1e-6, rope_theta=1e6, **common)
        hf = transformers.Qwen3ForCausalLM(hf_cfg)
        scaling, qk_norm, eps, theta = None, True, 1e-6, 1e6
    else:
        rs = {"rope_type": "llama3", "factor": 32.0, "low_freq_factor": 1.0,
              "high_freq_factor": 4.0, "original_max_position_embeddings": 64}
        hf_cfg = transformers.LlamaConfig(rms_norm_eps=1e-5, rope_theta=5e5, rope_scaling=rs,
                                          **common)
        hf = transformers.LlamaForCausalLM(hf_cfg)
        scaling = svllm_ops.Llama3RopeScaling(32.0, 1.0, 4.0, 64)
        qk_norm, eps, theta = False, 1e-5, 5e5
    hf = hf.to(device=device, dtype=torch.bfloat16).eval()
    cfg = svllm_ops.ModelConfig(vocab_size=VOCAB, hidden_size=HIDDEN, intermediate_size=INTER,
                                num_layers=LAYERS, num_heads=HEADS, num_kv_heads=KV_HEADS,
                                head_dim=HEAD_DIM, rms_norm_eps=eps, rope_theta=theta,
                                tie_word_embeddings=True, qk_norm=qk_norm, rope_scaling=scaling)
    model = svllm_ops.Model(cfg, dict(hf.state_dict()))
    model.allocate_kv_cache(64, BLOCK)
    return hf, model


class Requests:
    """Token histories and block tables of a few requests (blocks handed out out of order)."""

    def __init__(self, prompts: list[torch.Tensor], device: torch.device, blocks_per_req: int = 8):
        self.tokens = [p.clone() for p in prompts]
        order = torch.randperm(64, generator=torch.Generator().manual_seed(5))
        self.tables = order[: len(prompts) * blocks_per_req].view(len(prompts), blocks_per_req)
        self.tables = self.tables.to(torch.int32)
        self.cached = [0] * len(prompts)  # tokens already in the KV cache
        self.device = device

    def step_inputs(self, new: list[torch.Tensor]):
        """Inputs of one forward step that appends new[s] to request s."""
        ids, pos, slots, qsl = [], [], [], [0]
        for s, toks in enumerate(new):
            p = torch.arange(self.cached[s], self.cached[s] + len(toks))
            ids.append(toks)
            pos.append(p)
            slots.append(self.tables[s].long()[p // BLOCK] * BLOCK + p % BLOCK)
            qsl.append(qsl[-1] + len(toks))
            self.cached[s] += len(toks)
        d = self.device
        return dict(ids=torch.cat(ids).to(d), positions=torch.cat(pos).to(d),
                    slot_mapping=torch.cat(slots).to(d), block_tables=self.tables.to(d),
                    seq_lens=torch.tensor(self.cached, dtype=torch.int32, device=d),
                    query_start_loc=torch.tensor(qsl, dtype=torch.int32, device=d))


def hf_last_logits(hf, tokens: torch.Tensor, count: int, device) -> torch.Tensor:
    with torch.no_grad():
        return hf(tokens.to(device)[None]).logits[0, -count:].float()


def check_logits(ours: torch.Tensor, ref: torch.Tensor) -> None:
    ours = ours.float()
    bar = REL_BAR * ref.abs().max().item()
    assert (ours - ref).abs().max().item() <= bar
    top2 = ref.topk(2, dim=-1).values
    clear = (top2[:, 0] - top2[:, 1]) > bar
    assert torch.equal(ours.argmax(-1)[clear], ref.argmax(-1)[clear])


@pytest.mark.parametrize("arch", ["qwen3", "llama"])
def test_prefill_then_decode_matches_hugging_face(device, arch):
    hf, model = tiny(arch, device)
    g = torch.Generator().manual_seed(11)
    prompts = [torch.randint(0, VOCAB, (n,), generator=g) for n in (37, 20, 1)]
    reqs = Requests(prompts, device)
    # prefill all three requests in one packed step
    inputs = reqs.step_inputs(prompts)
    hidden = model.forward(**inputs)
    logits = model.logits(hidden)
    ends = inputs["query_start_loc"].tolist()
    for s, p in enumerate(prompts):
        check_logits(logits[ends[s]:ends[s + 1]], hf_last_logits(hf, p, len(p), device))
    last = torch.stack([logits[ends[s + 1] - 1] for s in range(3)]).float().argmax(-1).cpu()
    # three decode steps: one new token per request
    for _ in range(3):
        new = [last[s:s + 1] for s in range(3)]
        for s in range(3):
            reqs.tokens[s] = torch.cat([reqs.tokens[s], new[s]])
        inputs = reqs.step_inputs(new)
        hidden = model.forward(**inputs)
        ref = torch.cat([hf_last_logits(hf, reqs.tokens[s], 1, device) for s in range(3)])
        check_logits(model.logits(hidden), ref)
        ids = model.greedy(hidden)
        assert ids.dtype == torch.int64 and ids.device.type == device.type
        assert torch.equal(ids, model.logits(hidden).float().argmax(-1))
        last = ids.cpu()


def test_mixed_step_prefill_and_decode(device):
    """One step where one request decodes while another prefills a chunk of its prompt."""
    hf, model = tiny("qwen3", device)
    g = torch.Generator().manual_seed(12)
    a = torch.randint(0, VOCAB, (30,), generator=g)
    b = torch.randint(0, VOCAB, (25,), generator=g)
    reqs = Requests([a, b[:10]], device)
    model.forward(**reqs.step_inputs([a, b[:10]]))
    nxt = torch.tensor([7])
    reqs.tokens[0] = torch.cat([a, nxt])
    inputs = reqs.step_inputs([nxt, b[10:]])  # query lengths 1 and 15
    logits = model.logits(model.forward(**inputs))
    check_logits(logits[:1], hf_last_logits(hf, reqs.tokens[0], 1, device))
    check_logits(logits[1:], hf_last_logits(hf, b, 15, device))


def test_decode_entry_point_equals_forward_then_greedy(device):
    """decode() is forward() + greedy() for one-token steps. On CUDA its attention is the paged
    decode kernel instead of the gather + SDPA composite, so the ids must agree wherever the
    composite's top two logits differ by more than the bar."""
    _, model = tiny("qwen3", device)
    g = torch.Generator().manual_seed(13)
    prompts = [torch.randint(0, VOCAB, (n,), generator=g) for n in (9, 17)]
    reqs = Requests(prompts, device)
    model.forward(**reqs.step_inputs(prompts))
    inputs = reqs.step_inputs([torch.tensor([3]), torch.tensor([4])])
    qsl = inputs.pop("query_start_loc")
    assert qsl.tolist() == [0, 1, 2]
    logits = model.logits(model.forward(query_start_loc=qsl, **inputs)).float()
    got = model.decode(**inputs)
    if device.type == "cpu":
        assert torch.equal(got, model.greedy(model.forward(query_start_loc=qsl, **inputs)))
    top2 = logits.topk(2, dim=-1).values
    clear = (top2[:, 0] - top2[:, 1]) > REL_BAR * logits.abs().max()
    assert torch.equal(got[clear], logits.argmax(-1)[clear])


def test_padding_slot_writes_nothing(device):
    _, model = tiny("qwen3", device)
    before = [k.clone() for k in model.k_cache]
    ids = torch.tensor([5], device=device)
    one = dict(positions=torch.tensor([0], device=device),
               slot_mapping=torch.tensor([-1], device=device),
               block_tables=torch.zeros(1, 1, dtype=torch.int32, device=device),
               seq_lens=torch.ones(1, dtype=torch.int32, device=device))
    model.decode(ids, **one)
    for k0, k1 in zip(before, model.k_cache):
        assert torch.equal(k0, k1)


def test_errors_name_the_problem():
    hf, _ = tiny("qwen3", torch.device("cpu"))
    cfg = svllm_ops.ModelConfig(vocab_size=VOCAB, hidden_size=HIDDEN, intermediate_size=INTER,
                                num_layers=LAYERS, num_heads=HEADS, num_kv_heads=KV_HEADS,
                                head_dim=HEAD_DIM, rms_norm_eps=1e-6, rope_theta=1e6,
                                tie_word_embeddings=True, qk_norm=True)
    weights = dict(hf.state_dict())
    del weights["model.layers.1.mlp.up_proj.weight"]
    with pytest.raises(RuntimeError, match="missing weight model.layers.1.mlp.up_proj.weight"):
        svllm_ops.Model(cfg, weights)
    weights = dict(hf.state_dict())
    weights["model.norm.weight"] = weights["model.norm.weight"][:-1]
    with pytest.raises(RuntimeError, match="model.norm.weight has shape"):
        svllm_ops.Model(cfg, weights)
    model = svllm_ops.Model(cfg, dict(hf.state_dict()))
    z = torch.zeros(1, dtype=torch.long)
    with pytest.raises(RuntimeError, match="allocate_kv_cache first"):
        model.forward(z, z, z, torch.zeros(1, 1, dtype=torch.int32),
                      torch.ones(1, dtype=torch.int32), torch.tensor([0, 1], dtype=torch.int32))


# ---------------------------------------------------------------------------------------------
# decode steps replayed from CUDA graphs

def decode_batch(n: int, device, seed: int):
    """Inputs of a decode step for n requests with random histories already in the cache."""
    g = torch.Generator().manual_seed(seed)
    seq_lens = torch.randint(1, 8 * BLOCK, (n,), generator=g, dtype=torch.int32)
    pos = seq_lens.long() - 1
    # history blocks at random; the block each request writes to is its own
    tables = torch.randint(0, 64, (n, 8), generator=g)
    own = torch.randperm(64, generator=g)[:n]
    tables[torch.arange(n), pos // BLOCK] = own
    tables = tables.to(torch.int32)
    slots = own * BLOCK + pos % BLOCK
    ids = torch.randint(0, VOCAB, (n,), generator=g)
    return dict(ids=ids.to(device), positions=pos.to(device), slot_mapping=slots.to(device),
                block_tables=tables.to(device), seq_lens=seq_lens.to(device))


def padded(batch: dict, b: int) -> dict:
    """The same step padded to b requests the way DecodeGraphs pads."""
    n = batch["ids"].numel()
    if b == n:
        return batch
    d = batch["ids"].device
    pad = b - n
    return dict(ids=torch.cat([batch["ids"], torch.zeros(pad, dtype=torch.long, device=d)]),
                positions=torch.cat([batch["positions"],
                                     torch.zeros(pad, dtype=torch.long, device=d)]),
                slot_mapping=torch.cat([batch["slot_mapping"],
                                        torch.full((pad,), -1, dtype=torch.long, device=d)]),
                block_tables=torch.cat([batch["block_tables"],
                                        torch.zeros(pad, batch["block_tables"].size(1),
                                                    dtype=torch.int32, device=d)]),
                seq_lens=torch.cat([batch["seq_lens"],
                                    torch.ones(pad, dtype=torch.int32, device=d)]))


@pytest.mark.gpu
def test_decode_graph_buckets(cuda):
    _, model = tiny("qwen3", cuda)
    # fill every block with random history so attention reads real values
    for k, v in zip(model.k_cache, model.v_cache):
        k.normal_(generator=torch.Generator(device=cuda).manual_seed(1))
        v.normal_(generator=torch.Generator(device=cuda).manual_seed(2))
    graphs = svllm_ops.DecodeGraphs(model, max_num_seqs=24, max_blocks_per_seq=8)
    assert graphs.batch_sizes == [1, 2, 4, 8, 16, 24]
    for n, seed in [(1, 1), (3, 2), (8, 3), (13, 4), (24, 5), (3, 6)]:
        batch = decode_batch(n, cuda, seed)
        b = min(s for s in graphs.batch_sizes if s >= n)
        caches = [k.clone() for k in model.k_cache]
        got = graphs.step(**batch)
        graph_caches = [k.clone() for k in model.k_cache]
        for k, c in zip(model.k_cache, caches):
            k.copy_(c)
        want = model.decode(**padded(batch, b))[:n]
        assert torch.equal(got, want), (n, b)
        for k, c in zip(model.k_cache, graph_caches):
            assert torch.equal(k, c)


@pytest.mark.gpu
def test_decode_graph_rejects_oversized_batches(cuda):
    _, model = tiny("qwen3", cuda)
    graphs = svllm_ops.DecodeGraphs(model, max_num_seqs=4, max_blocks_per_seq=2,
                                    batch_sizes=[4, 2])
    assert graphs.batch_sizes == [2, 4]
    with pytest.raises(RuntimeError, match="largest captured batch is 4"):
        graphs.step(**decode_batch(5, cuda, 0))
    with pytest.raises(RuntimeError, match="block tables of at most 2"):
        graphs.step(**decode_batch(2, cuda, 0))


def test_decode_graphs_need_cuda():
    _, model = tiny("qwen3", torch.device("cpu"))
    with pytest.raises(RuntimeError, match="CUDA graphs need a model on a CUDA device"):
        svllm_ops.DecodeGraphs(model, max_num_seqs=4, max_blocks_per_seq=2)
