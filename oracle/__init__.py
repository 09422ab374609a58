"""CPU oracle for lightserve's attention hot path -- TEST INFRASTRUCTURE ONLY.

A restatement, in numpy/PyTorch-CPU, of the algorithms the reference runs on
this path. It exists to check the CUDA kernels of ``lightserve_b200`` and to
time the reference's CPU path beside them. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its CPU baseline leg and its
``--impl reference`` arm) may import it; the ``lightserve_b200`` package never
does, and never falls back to it.

Pinning: every function here is checked against golden vectors produced by
lightserve's own code (its Triton kernels run by the Triton CPU interpreter in
fp32, and its ``reference_llama_forward`` greedy decode), committed under
``tests/golden/`` together with the script that generated them
(``tests/golden/make_golden.py``).
"""
