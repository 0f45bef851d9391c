"""rollout"""
