"""CPU oracle of the PLM decoding round — TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, what the reference (justuswill/PLM-anon) computes on the round's hot path. It
exists to check the CUDA kernels of ``plm-anon_b200``; nothing in the product imports it. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may use it.

Modules
  exact    float32 arithmetic with a fully specified operation order (elementary functions, reductions) shared by
           definition with the GPU kernels, so verify decode and acceptance can be compared bit for bit.
  voronoi  plm/iterate.py (the Voronoi assignment engine) and the acceptance rules of plm/decoder.py:71-82.
  model    the Llama forward of vLLM's model (RMSNorm, neox RoPE, SiLU-gated MLP) over a paged KV cache, the round
           layout and mask (plm/mask.py), and the RoundDecoder state machine (plm/decoder.py:275-467).
  ptp      the gated-LoRA model's PTP scheme (plm/auxiliary.py:78-113, plm/gated_lora.py:35-90): blended auxiliary
           inputs, the inverse-CDF verify decode and adapters on the gated rows.

Parity pins (see tests/golden/make_golden.py): the reference's own functions, run on CPU in the build container
(Triton kernels under TRITON_INTERPRET=1, the prologue/epilogue methods called on CPU tensors), and Hugging Face
transformers' LlamaForCausalLM for the forward.
"""
