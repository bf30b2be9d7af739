"""Expert parallelism: fused NVLink dispatch/combine, placement planner, speculative replicas,
two-stage path, symmetric buffers."""
