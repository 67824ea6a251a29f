"""CPU oracle for the sparse paged GQA FP8 decode-attention path.

TEST INFRASTRUCTURE ONLY. Nothing in the product (the ``qsa_b200`` package,
its C-ABI library or its torch extension) imports or calls this package.
Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` use it, and only as the checker
or as the timed CPU baseline -- never as the thing measured or shipped.

Modules:

* ``qsa_oracle`` -- numpy restatement of the reference's eager path
  (``sm89_torch.py:27-54``) and of its loop reference
  (``sm89_cutedsl.py:83-116``), plus the slot-addressing oracle used for the
  bit-exact check. Parity is pinned against golden vectors produced by the
  reference itself (``tests/golden/make_golden.py``).
* ``eager_port`` -- the same eager algorithm expressed with the same ATen
  operators on CPU tensors; it is what the CPU baseline times.
* ``build_ref.sh`` -- compiles the reference's own CUDA kernel
  (``sm89_cuda.cu``) for sm_100a into ``oracle/_ref/`` as a GPU comparator.
"""
