"""Record what the REFERENCE's ``apply_to`` does with the synthetic containers of
tests/ebin_synth.py, as tests/golden/loader_<levels>.json.

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_loader_golden.py /path/to/epure-runtime

Imports the reference package ``epure`` from that checkout, swaps its
``container.rans_decode`` for the identity decoder (the synthetic index streams
are stored raw; ``constriction`` is not installed), loads each container into
the toy module tree with ``apply_to`` (epure/runtime.py:214-305) and records:

* the class of every module and the shape of every parameter afterwards (the
  module-swap rules: embedding, linear, convolution, expert slab, router);
* float64 sums of every dense parameter and of every packed module's
  ``materialize(float32)`` / PackedLinear output on a fixed input (values);
* whether the tied lm_head shares the embedding's store, and the config flag.

tests/test_loader.py compares the repository's ``apply_to`` against these.
"""
import json
import os
import sys
import tempfile


def main(ref_root):
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.dirname(here))        # tests/ (ebin_synth)
    sys.path.insert(0, ref_root)                     # the reference's epure package
    import torch
    import ebin_synth as S
    from epure import container, runtime

    container.rans_decode = S.identity_decode
    for levels in (16, 256):
        with tempfile.TemporaryDirectory() as d:
            path = os.path.join(d, "toy.ebin")
            S.make_container(path, levels=levels, group=16)
            model = S.toy_model()
            runtime.apply_to(model, path, device="cpu", cfg=model.config, verbose=False,
                             dtype=torch.float32)
        x = torch.linspace(-1, 1, 32)
        rec = {"structure": S.describe_model(model),
               "tie_flag": bool(model.config.tie_word_embeddings),
               "lm_head_is_embedding_store": model.lm_head.store is model.model.embed_tokens.store,
               "dense_sums": {n: float(p.double().sum()) for n, p in model.named_parameters()},
               "q_proj_out_sum": float(model.model.layers[0].self_attn.q_proj(x[None]).double().sum()),
               "embed_rows_sum": float(model.model.embed_tokens(torch.tensor([[1, 5, 63]])).double().sum()),
               "lm_head_out_sum": float(model.lm_head(x[None]).double().sum())}
        with open(os.path.join(here, f"loader_l{levels}.json"), "w") as f:
            json.dump(rec, f, indent=1, sort_keys=True)
        print(f"loader_l{levels}.json: {len(rec['structure'])} entries")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_loader_golden.py <path to the epure-runtime checkout>")
    main(sys.argv[1])
