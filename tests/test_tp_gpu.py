"""Tensor-parallel decoder on the GPU, loaded from a compressed store: one
GPU (decoded and compressed-resident shards) and, when two GPUs are
present, two NCCL ranks -- logits within BF16 tolerance of a plain
transformers forward, greedy tokens equal where the top-2 margin is clear."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from bf16tol import FUSED_STEP_ATOL, check_logits
from test_streaming_engine_gpu import _store, _tiny

pytestmark = pytest.mark.gpu


def _ref_greedy(model, ids, n):
    seq = ids
    margins = []
    with torch.no_grad():
        for _ in range(n):
            lg = model(input_ids=seq).logits[0, -1].float()
            top = torch.topk(lg, 2).values
            margins.append(float(top[0] - top[1]))
            seq = torch.cat([seq, lg.argmax().reshape(1, 1)], 1)
    return seq, margins


def _check_single_token_steps(dec, model, ids, n):
    """The decoder's single-token steps against transformers' own KV-cache
    steps, fed the same tokens: logits within 1e-2 (or one BF16 rounding
    step) at every step for the unfused torch math, within FUSED_STEP_ATOL
    for the fused layer kernels."""
    from afterimage_b200.runtime.tp_decoder import KVCache
    cache = KVCache(dec.n_layers, dec.nkv, dec.hd, ids.shape[1] + n + 2, dec.device)
    pkv = None
    step = ids
    with torch.no_grad():
        for _ in range(n):
            out = model(input_ids=step, past_key_values=pkv, use_cache=True)
            pkv = out.past_key_values
            ref = out.logits[0, -1].float()
            got = dec.forward(step, cache)[-1].float()
            check_logits(got, ref, atol=FUSED_STEP_ATOL if dec.fused else 1e-2)
            step = ref.argmax().reshape(1, 1)


def _check_greedy(seq, ref_seq, margins, n_prompt):
    for t, mg in enumerate(margins):
        if mg > 0.05:
            assert int(seq[0, n_prompt + t]) == int(ref_seq[0, n_prompt + t])
        else:
            break  # after a near-tie the continuations may legitimately differ


@pytest.fixture(scope="module")
def stores(tmp_path_factory):
    from afterimage_b200.runtime.streaming_engine import write_store
    tmp = tmp_path_factory.mktemp("tp")
    cfg, model = _tiny(tie=False, seed=21, layers=2)
    snap, store, _ = _store(tmp, cfg, model, "ref")  # reference chunking (256)
    tp_store = tmp / "tp_ready"
    write_store(((k, v.contiguous()) for k, v in model.state_dict().items()), tp_store, tied=False,
                tp_row_chunks=4)
    return cfg, model, store, tp_store


@pytest.mark.parametrize("resident,kw", [("decoded", {}), ("compressed", {}),
                                         ("compressed", {"overlap": True, "head_block_rows": 500}),
                                         ("streamed", {}), ("streamed", {"slots": 3, "overlap": True}),
                                         ("streamed", {"slots": 1, "head_block_rows": 1536}),
                                         ("decoded", {"fused": False}), ("streamed", {"fused": False})])
@pytest.mark.parametrize("which", ["ref", "tp_ready"])
def test_tp_single_gpu_matches_transformers(stores, resident, kw, which):
    from afterimage_b200.runtime.tp_decoder import load_tp_decoder
    cfg, model, store, tp_store = stores
    dec = load_tp_decoder(store if which == "ref" else tp_store, cfg, 1, 0, None, "cuda", resident=resident, **kw)
    model = model.to("cuda")
    ids = torch.randint(0, cfg.vocab_size, (1, 11), device="cuda")
    with torch.no_grad():
        ref = model(input_ids=ids).logits[0].float()
    got = dec.forward(ids).float()
    check_logits(got, ref)
    _check_single_token_steps(dec, model, ids, 4)
    seq = dec.generate_greedy(ids, 5)
    ref_seq, margins = _ref_greedy(model, ids, 5)
    _check_greedy(seq, ref_seq, margins, 11)
    if resident != "decoded":
        _lib_status_clear()
    if resident == "streamed":
        assert dec.h2d_bytes > 0
        dec.close()


@pytest.fixture(scope="module")
def tied_store(tmp_path_factory):
    from afterimage_b200.runtime.streaming_engine import write_store
    tmp = tmp_path_factory.mktemp("tp_tied")
    cfg, model = _tiny(tie=True, seed=22, layers=2)
    items = ((k, v.contiguous()) for k, v in model.state_dict().items() if k != "lm_head.weight")
    write_store(items, tmp / "tied", tied=True, tp_row_chunks=4)
    return cfg, model, tmp / "tied"


@pytest.mark.parametrize("resident,kw", [("decoded", {}), ("compressed", {}), ("streamed", {}),
                                         ("streamed", {"vram_budget_gb": 100.0})])
def test_tp_tied_head_matches_transformers(tied_store, resident, kw):
    """A tied checkpoint (no lm_head.weight in the store): the head is this
    rank's vocabulary rows of the embedding, in every residency mode, eager
    and graphed."""
    from afterimage_b200.runtime.tp_decoder import load_tp_decoder
    cfg, model, store = tied_store
    dec = load_tp_decoder(store, cfg, 1, 0, None, "cuda", resident=resident, **kw)
    model = model.to("cuda")
    ids = torch.randint(0, cfg.vocab_size, (1, 10), device="cuda",
                        generator=torch.Generator(device="cuda").manual_seed(8))
    with torch.no_grad():
        ref = model(input_ids=ids).logits[0].float()
    got = dec.forward(ids).float()
    check_logits(got, ref)
    _check_single_token_steps(dec, model, ids, 4)
    ref_seq, margins = _ref_greedy(model, ids, 5)
    _check_greedy(dec.generate_greedy(ids, 5), ref_seq, margins, 10)
    if resident != "streamed":
        _check_greedy(dec.generate_greedy_graphed(ids, 5), ref_seq, margins, 10)
    if resident != "decoded":
        _lib_status_clear()
    dec.close()


@pytest.mark.parametrize("resident,kw", [("decoded", {}), ("compressed", {}), ("compressed", {"overlap": True}),
                                         ("decoded", {"fused": False}), ("compressed", {"fused": False})])
def test_tp_graphed_generation(stores, resident, kw):
    """The single-token step captured as a CUDA graph (decode launches
    included) gives the greedy tokens of the eager decoder and of
    transformers; a second call replays the same graph."""
    from afterimage_b200.runtime.tp_decoder import load_tp_decoder
    cfg, model, store, tp_store = stores
    dec = load_tp_decoder(tp_store, cfg, 1, 0, None, "cuda", resident=resident, **kw)
    model = model.to("cuda")
    for seed, P in ((3, 9), (4, 9), (5, 12), (6, 9)):
        ids = torch.randint(0, cfg.vocab_size, (1, P), device="cuda",
                            generator=torch.Generator(device="cuda").manual_seed(seed))
        seq = dec.generate_greedy_graphed(ids, 6)
        eager = dec.generate_greedy(ids, 6)
        ref_seq, margins = _ref_greedy(model, ids, 6)
        _check_greedy(seq, ref_seq, margins, P)
        _check_greedy(seq, eager, margins, P)
        assert seq.shape == (1, P + 6)
    st = dec._graph_state
    assert st is not None and st.graph is not None and sorted(st.prefill) == [9, 12]
    if resident != "decoded":
        _lib_status_clear()
    dec.close()


def test_tp_streamed_under_a_per_rank_budget(stores):
    """A per-rank VRAM budget keeps the layers the planner picks resident in
    HBM and streams only the rest; weights and tokens are unchanged."""
    from afterimage_b200.runtime.tp_decoder import load_tp_decoder
    cfg, model, store, tp_store = stores
    big = load_tp_decoder(tp_store, cfg, 1, 0, None, "cuda", resident="streamed", vram_budget_gb=100.0)
    assert big.streamed == [] and big.h2d_bytes_per_forward() == 0
    fixed = big.budget_plan["fixed_bytes"]
    one = big.images[0].numel()
    big.close()
    dec = load_tp_decoder(tp_store, cfg, 1, 0, None, "cuda", resident="streamed",
                          vram_budget_gb=(fixed + one + 1000) / 1e9)
    assert sorted(dec.images) == [0] and dec.streamed == list(range(1, cfg.num_hidden_layers))
    sd = {k: v.to("cuda") for k, v in model.state_dict().items()}
    for rep in range(2):
        for i in range(cfg.num_hidden_layers):
            for name, w in dec.layer_weights(i).items():
                if name in ("self_attn.qkv_proj.weight", "mlp.gate_up_proj.weight"):
                    continue
                assert torch.equal(w.view(torch.int16), sd["model.layers.%d.%s" % (i, name)].view(torch.int16))
    model = model.to("cuda")
    ids = torch.randint(0, cfg.vocab_size, (1, 7), device="cuda")
    seq = dec.generate_greedy(ids, 4)
    ref_seq, margins = _ref_greedy(model, ids, 4)
    _check_greedy(seq, ref_seq, margins, 7)
    assert dec.h2d_bytes_per_forward() == sum(int(h.numel()) for h in dec.host.values()) > 0
    dec.close()


def _lib_status_clear():
    from afterimage_b200.runtime import _device
    _device.check_status(torch.device("cuda", torch.cuda.current_device()))


def test_tp_decoded_weights_bit_exact(stores):
    """The compressed and streamed decoders produce exactly the weights of
    the plain decode (every layer, every shard)."""
    from afterimage_b200.runtime.tp_decoder import load_tp_decoder
    cfg, model, store, tp_store = stores
    sd = {k: v.to("cuda") for k, v in model.state_dict().items()}
    for path in (store, tp_store):
        for resident in ("compressed", "streamed"):
            dec = load_tp_decoder(path, cfg, 1, 0, None, "cuda", resident=resident)
            for rep in range(2):  # second pass: the streamed ring wraps around
                for i in range(cfg.num_hidden_layers):
                    W = dec.layer_weights(i)
                    for name, w in W.items():
                        key = "model.layers.%d.%s" % (i, name)
                        if name in ("self_attn.qkv_proj.weight", "mlp.gate_up_proj.weight"):
                            parts = ("q_proj", "k_proj", "v_proj") if "qkv" in name else ("gate_proj", "up_proj")
                            pre = key.rsplit(".", 2)[0]
                            want = torch.cat([sd["%s.%s.weight" % (pre, n)] for n in parts], 0)
                        else:
                            want = sd[key]
                        assert torch.equal(w.view(torch.int16), want.view(torch.int16)), name
            if resident == "streamed":
                dec.close()


def _rank_main(rank, world, port, tp_store, cfg_dict, ids, q, resident):
    from transformers import Qwen3Config
    from afterimage_b200.runtime.tp_decoder import load_tp_decoder
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    torch.distributed.init_process_group("nccl", rank=rank, world_size=world,
                                         timeout=datetime.timedelta(seconds=120),
                                         device_id=torch.device("cuda", rank))
    try:
        cfg = Qwen3Config(**cfg_dict)
        dec = load_tp_decoder(tp_store, cfg, world, rank, None, "cuda:%d" % rank, resident=resident)
        logits = dec.forward(ids.to("cuda:%d" % rank)).float().cpu().numpy()
        seq = dec.generate_greedy(ids.to("cuda:%d" % rank), 5).cpu().numpy()
        gseq = dec.generate_greedy_graphed(ids.to("cuda:%d" % rank), 5).cpu().numpy() \
            if resident != "streamed" else seq
        dec.release_graphs()
        q.put((rank, logits, seq, gseq))
        if resident == "streamed":
            dec.close()
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("resident", ["compressed", "streamed"])
def test_tp_two_gpus_nccl_matches_transformers(stores, resident):
    cfg, model, store, tp_store = stores
    ids = torch.randint(0, cfg.vocab_size, (1, 11))
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, str(tp_store), cfg.to_dict(), ids, q, resident)) for r in range(2)]
    for p in procs:
        p.start()
    got = sorted([q.get(timeout=300) for _ in range(2)], key=lambda g: g[0])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    model = model.to("cuda:0")
    with torch.no_grad():
        ref = model(input_ids=ids.to("cuda:0")).logits[0].float().cpu()
    for rank, logits, seq, gseq in got:
        logits = torch.from_numpy(logits)
        check_logits(logits, ref)
    ref_seq, margins = _ref_greedy(model, ids.to("cuda:0"), 5)
    _check_greedy(torch.from_numpy(got[0][2]), ref_seq.cpu(), margins, 11)
    _check_greedy(torch.from_numpy(got[0][3]), ref_seq.cpu(), margins, 11)
    assert (got[0][3] == got[1][3]).all()  # ranks agree


@pytest.mark.parametrize("resident", ["compressed", "streamed"])
def test_tp_speculative_decoding_equals_greedy_on_gpu(stores, resident):
    """Draft/target speculation in the tensor-parallel decoder at temperature
    0 (reference streaming_engine.py:2488-2575): the compressed or streamed
    target verifies k proposals in one (k+1)-token forward; the tokens are
    the target's greedy tokens wherever its top-2 margin is clear, for an
    unrelated random draft and for the target as its own draft (whose
    proposals are accepted)."""
    from afterimage_b200.runtime.tp_decoder import TPDecoder, load_tp_decoder
    cfg, model, store, tp_store = stores
    dec = load_tp_decoder(tp_store, cfg, 1, 0, None, "cuda", resident=resident)
    _, other = _tiny(tie=False, seed=77, layers=2)
    unrelated = TPDecoder(cfg, {k: v.to("cuda") for k, v in other.state_dict().items()}, 1, 0, None, "cuda")
    itself = load_tp_decoder(tp_store, cfg, 1, 0, None, "cuda", resident="decoded")
    ids = torch.randint(0, cfg.vocab_size, (1, 9), device="cuda", generator=torch.Generator(device="cuda").manual_seed(3))
    ref_seq, margins = _ref_greedy(model.to("cuda"), ids, 8)
    for draft, k in ((unrelated, 3), (itself, 4)):
        st = {}
        seq = dec.generate_speculative(ids, 8, draft, k=k, stats=st)
        assert seq.shape == (1, 17)
        _check_greedy(seq, ref_seq, margins, 9)
        if draft is itself:
            assert st["accepted_from_draft"] >= 4 and st["sweeps"] <= 4
    if resident == "streamed":
        dec.close()


def test_tp_wide_projections_on_own_kernels_match_transformers(tmp_path, monkeypatch):
    """gate/up (2 x 8192 rows) and the head (16384 rows) are wide enough for
    the fused mode to route them to this package's GEMV (up to 8 tokens) and
    tcgen05 GEMM (9-64 tokens): logits for 1, 5, 11 and 70 tokens stay within
    the BF16 tolerance of transformers, and both kernels are really used."""
    from transformers import AutoModelForCausalLM, Qwen3Config
    from afterimage_b200.runtime import tp_ops
    from afterimage_b200.runtime.streaming_engine import write_store
    from afterimage_b200.runtime.tp_decoder import TPDecoder, load_tp_decoder
    torch.manual_seed(5)
    cfg = Qwen3Config(vocab_size=16384, hidden_size=320, intermediate_size=8192, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=80, max_position_embeddings=256,
                      tie_word_embeddings=False)
    model = AutoModelForCausalLM.from_config(cfg, dtype=torch.bfloat16)
    with torch.no_grad():
        for p in model.parameters():
            if p.dim() == 2:
                p.normal_(0, 0.02)
    model = model.eval()
    store = tmp_path / "wide"
    write_store(((k, v.contiguous()) for k, v in model.state_dict().items()), store, tied=False)
    assert 2 * cfg.intermediate_size >= TPDecoder.OWN_KERNEL_MIN_ROWS
    calls = {"gemv": 0, "gemm_tc": 0}
    for name in calls:
        real = getattr(tp_ops, name)

        def counted(*a, _real=real, _name=name, **k):
            calls[_name] += 1
            return _real(*a, **k)
        monkeypatch.setattr(tp_ops, name, counted)
    dec = load_tp_decoder(store, cfg, 1, 0, None, "cuda", resident="decoded")
    model = model.to("cuda")
    g = torch.Generator(device="cuda").manual_seed(9)
    for T in (5, 11, 70):
        ids = torch.randint(0, cfg.vocab_size, (1, T), device="cuda", generator=g)
        with torch.no_grad():
            ref = model(input_ids=ids).logits[0].float()
        check_logits(dec.forward(ids).float(), ref)
    assert calls["gemv"] > 0 and calls["gemm_tc"] > 0
    # single-token steps after an 11-token prompt (fused layer kernels + GEMV)
    ids = torch.randint(0, cfg.vocab_size, (1, 11), device="cuda", generator=g)
    _check_single_token_steps(dec, model, ids, 4)
