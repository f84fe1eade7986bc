"""Component benchmarks: rollout-only throughput, train-step throughput,
weight-sync latency vs NVLink roofline, collective bandwidth (C38)."""
