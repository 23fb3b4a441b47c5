"""gpt-oss MXFP4 MoE block and sink/YaRN attention on B200 (sm_100a)."""
