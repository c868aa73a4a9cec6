"""Accuracy-gate calibration faults (reference ``model.py:149-173``, ``server.py:780-840``).

Each fault deliberately breaks one piece of the model so an accuracy checker can be shown to
catch it; all are off unless set, and are switched at runtime through ``POST /debug/fault``
(enabled with ``QB_FAULT_ENDPOINT=1``) or by setting ``Model.fault[name]`` directly. They act
on the host side of the model (which arguments the kernels receive); none of them makes a GPU
kernel fault or hang.

* ``rope_base``          - RoPE theta used by the attention layers (a wrong base)
* ``drop_expert``        - zero the routing weight of one expert id
* ``skip_deltanet_gate`` - replace the DeltaNet gated output norm by a plain RMSNorm
* ``fp8_kv_no_scale``    - round every new K/V cache row through e4m3 with no scale factor
* ``flip_causal_mask``   - one full-attention layer attends bidirectionally within the context
                           (its prefill queries also see later keys of their segment)
* ``flip_causal_mask_layer`` - which full-attention layer (0-based among full-attention layers)

While any fault is set, decode and speculative rounds run eagerly instead of replaying their
captured graphs (a graph holds the kernels' arguments of its capture).
"""

FAULTS = {"rope_base", "drop_expert", "skip_deltanet_gate", "fp8_kv_no_scale", "flip_causal_mask",
          "flip_causal_mask_layer"}
