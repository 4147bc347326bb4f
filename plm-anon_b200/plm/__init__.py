"""B200-native PLM decoding round: the host side of libplm_native.so.

Mirrors the reference's ``plm`` package entry points (``plm.rounds.RoundConfig``, ``plm.decoder.RoundDecoder``,
``plm.mask.round_layout``) over hand-written sm_100a kernels. Nothing here imports vLLM or Triton.
"""
