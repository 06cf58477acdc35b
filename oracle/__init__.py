"""CPU oracle for the decode path -- TEST INFRASTRUCTURE ONLY.

Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
leg, as the checker and the timed CPU baseline; the product never imports it.
The reference's own golden vectors need real checkpoints that are absent from
its tree.  The oracle is pinned instead to the reference's golden generator:
the reference verifies its semantics against transformers' modeling_gemma4.py
(src/engine-a4b.js:1-11) and makes its goldens with transformers in f32
(goldens/gen.py).  With f32 storage (ops.STORE_F16 = False) the oracle
reproduces transformers' Gemma4ForCausalLM on seven synthetic models to 1e-4
(tests/test_pin_transformers.py, fixtures from tests/golden/make_pin.py); the
`gguf` package pins the block decoders (tests/test_oracle.py).
"""
