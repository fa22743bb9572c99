"""CPU oracle for the MoE + embedding-bag hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product (the ``cti_b200`` package,
its C ABI and kernels) imports, links or calls this package.  Only
``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / reference
leg of ``bench.py`` use it, always as the checker or the timed CPU baseline,
never as the thing measured or shipped.

Contents:
  moe_ref.py         restatement of the reference Top-2 MoE layer
                     (baseline/infer.py:280-358) in fp32 torch on CPU,
                     plus fp64 logits for the near-tie policy.
  embbag_ref.py      restatement of the reference embedding-bag pooling
                     (baseline/infer.py:253-263) in fp32 on CPU.
  router_order.c     the router restated in C with the kernel's fixed
                     reduction order (two fmaf chains per logit, even and
                     odd d, then the bias), for a strict bit-exact check
                     of expert indices.
  e2e_ref.py         the reference CTR model graph (baseline/infer.py:
                     244-439) in fp32 at the end-to-end configuration,
                     and its RepEncoder alone (rep_encoder_ref, :253-265).
  build.py           compiles router_order.c into _build/liborder.so.

Pinning: tests/golden/ holds fixtures produced by running the reference's
own code (tests/golden/make_golden.py imports baseline/infer.py); the tests
check this oracle against them.
"""
