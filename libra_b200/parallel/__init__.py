"""Model parallelism: rank mesh, tensor/sequence-free TP layers, pipeline schedule, expert parallelism."""
