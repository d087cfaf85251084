"""Collectives: the reference's Communicator API on NCCL over NVLink."""

from .communicator import Communicator, CommunicatorStats, ProcessGroup

__all__ = ["Communicator", "CommunicatorStats", "ProcessGroup"]
