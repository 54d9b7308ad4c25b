"""Reference (PyTorch) implementations of the other architectures the reference carries as
libraries (``src/mla.rs``, ``src/mamba.rs``, ``src/rwkv.rs``, ``src/gated_deltanet.rs``,
``src/yarn.rs``, ``src/gemma4.rs``, ``src/ops.rs`` variants). They are the numerics oracles a
fused sm_100a kernel for each would be tested against."""
