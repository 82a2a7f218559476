"""Elastic Hybrid Pool: borrowed rollout GPUs joining training as whole DP replicas."""

from libra_b200.infra.elastic.hybrid_pool import (DEFAULT_CHUNK_BYTES, ElasticHybridPool, ElasticWorker,
                                                  GradientCommunicationDomains, GradientPayload, GradientTransport,
                                                  InterReplicaGradientDomain, JoinCancelledError, JoinHandle,
                                                  JoinState, PeerMemoryTransport, ReplicaJoinHandle, ReplicaRole,
                                                  TorchDistributedRDMATransport, TorchDistributedTransport)

__all__ = ["DEFAULT_CHUNK_BYTES", "ElasticHybridPool", "ElasticWorker", "GradientCommunicationDomains",
           "GradientPayload", "GradientTransport", "InterReplicaGradientDomain", "JoinCancelledError", "JoinHandle",
           "JoinState", "PeerMemoryTransport", "ReplicaJoinHandle", "ReplicaRole", "TorchDistributedRDMATransport",
           "TorchDistributedTransport"]
