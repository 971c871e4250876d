"""Evidence and experiment harness.

Host-side tooling that turns runs into auditable evidence, with the same
capabilities as the reference's ``experiments/`` and ``eval/`` scripts:

=====================  ==========================================================
module                 what it does (reference counterpart)
=====================  ==========================================================
``bundle``             run one command into an immutable, checksummed bundle;
                       validate a bundle (run_experiment.py, validate_run_bundle.py)
``paired``             ABBA paired summaries of two variants (summarize_paired_results.py)
``kernels``            kernel-time classification of a launch list
                       (analyze_nsys_kernel_summary.py)
``rank_profile``       per-rank kernel profiles of a multi-rank job (profile_rank_with_nsys.py)
``contract``           parameter-name / QKV-layout / TP-shard contracts between this
                       framework, the reference and Megatron-Core
                       (fair_tp1_contract.py, fair_tp_parallel_contract.py)
``parity``             numerical parity gates: logits, loss, gradients, parameters
                       after one AdamW step (validate_mcore_equivalence.py,
                       validate_mcore_tp_equivalence.py, summarize_fair_pp_gate.py)
``artifacts``          freeze shared source weights, per-rank shards and fixed
                       next-token batches (create_fair_*_artifacts.py)
``fair_bench``         compute-only benchmark of one implementation on frozen
                       artifacts, with CUDA-event phase timing (run_fair_*_benchmark.py)
``queue``              sequential ABBA runner with an idle-GPU gate
                       (run_tp2_preliminary_queue.py, run_fair_pp_queue.py)
``campaign``           append-only evidence ledger with a publication rule
                       (fair_parallel_campaign.py)
``conclusions``        multi-window gate conclusions and profile indexes
                       (write_fair_pp_conclusion.py, summarize_fair_pp_profiles.py,
                       summarize_fair_pp_gate_windows.py)
``legacy``             synthetic / identity datasets, convergence and loss
                       comparisons, archived benchmark sweeps (synthetic_data.py,
                       make_identity.py, compare_convergence.py,
                       save_benchmark_results.py, eval/compare_loss.py)
``baselines``          external-framework baseline arms: the reference
                       mini-megatron and, when installed, Megatron-Core
                       (eval/run_megatron_baseline.py)
=====================  ==========================================================

Nothing here launches a GPU kernel of its own; GPU work happens in the
commands a bundle runs.  Profiling uses ``ncu`` launch lists (one pass) and
the PyTorch profiler, since Nsight Systems is not part of this toolchain.
"""
