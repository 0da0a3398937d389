"""CPU oracle for litevllm's per-step hot path — TEST INFRASTRUCTURE ONLY.

Plain restatements of the reference algorithms (lxy-alexander/lite-vllm,
paths relative to that project), used as the checker by tests/, by
__graft_entry__.smoke() and by bench.py's CPU-baseline / reference arm.
Nothing in the product (litevllm_b200/) imports this package.

  store_kv.py         KV store            litevllm/layers/attention.py:79-84, :18-33
  paged_attention.py  decode              litevllm/layers/attention.py:91-139
                      prefill (+prior)    litevllm/layers/attention.py:141-151 composed
                                          with the gather of :105-119
  sampler.py          greedy argmax       litevllm/layers/sampler.py:60-84, :174-175
                      Gumbel-max          restates :178, :187 (softmax(x/T) + draw) as
                                          argmax(x/T + g) for a given noise g
                      Philox4x32-10       the in-kernel noise generator, bit-exact ints

Pinning: tests/golden/ holds outputs of the reference's own functions,
imported from the reference checkout and run on CPU by
tests/golden/make_golden.py; tests/test_oracle_golden.py checks every
restatement here against them, and the four vectors of the reference's
tests/test_sampler.py are checked verbatim.
"""
