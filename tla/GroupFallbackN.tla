---------------------------- MODULE GroupFallbackN ----------------------------
(* One outer NCCL group seen by the interposer, for a clique of N ranks.     *)
(* Calls arrive one at a time: a collective of rank i ("r" \o i) or an       *)
(* unsupported operation. A rank call is buffered while nothing went         *)
(* passthrough and fewer than N calls are pending; otherwise the buffered    *)
(* prefix and the call are forwarded to libnccl, in order, and the group    *)
(* becomes passthrough. End runs the clique exactly when nothing went        *)
(* passthrough and the pending calls are one call of every rank.             *)
EXTENDS Naturals, Sequences, FiniteSets

CONSTANTS N, MaxCalls, SkipUnsupportedFlush
VARIABLES seen, forwarded, pending, passthrough, unsupported, ended, custom
vars == <<seen, forwarded, pending, passthrough, unsupported, ended, custom>>

Ranks == 0..(N - 1)
Ops == Ranks \cup {N}            \* N stands for "unsupported"
Range(s) == {s[i] : i \in 1..Len(s)}
Clique(s) == Len(s) = N /\ Range(s) = Ranks

Init == /\ seen = <<>> /\ forwarded = <<>> /\ pending = <<>>
        /\ passthrough = FALSE /\ unsupported = FALSE
        /\ ended = FALSE /\ custom = FALSE

Receive(op) ==
  /\ ~ended /\ Len(seen) < MaxCalls
  /\ seen' = Append(seen, op)
  /\ unsupported' = (unsupported \/ op = N)
  /\ IF op = N /\ SkipUnsupportedFlush
       THEN /\ forwarded' = Append(forwarded, op)
            /\ UNCHANGED <<pending, passthrough>>
       ELSE IF passthrough \/ op = N \/ Len(pending) = N
         THEN /\ forwarded' = Append(forwarded \o pending, op)
              /\ pending' = <<>> /\ passthrough' = TRUE
         ELSE /\ pending' = Append(pending, op)
              /\ UNCHANGED <<forwarded, passthrough>>
  /\ UNCHANGED <<ended, custom>>

End == /\ ~ended /\ ended' = TRUE
       /\ custom' = (~passthrough /\ Clique(pending))
       /\ forwarded' = IF ~passthrough /\ Clique(pending)
                         THEN forwarded ELSE forwarded \o pending
       /\ pending' = <<>>
       /\ UNCHANGED <<seen, passthrough, unsupported>>

Next == (\E op \in Ops : Receive(op)) \/ End
Spec == Init /\ [][Next]_vars

OrderedPrefix == /\ Len(forwarded) <= Len(seen)
                 /\ forwarded = SubSeq(seen, 1, Len(forwarded))
PendingBound == Len(pending) <= N
BufferedOrder == ~ended => forwarded \o pending = seen
Complete == ended => IF custom
                       THEN /\ Clique(seen) /\ ~unsupported /\ forwarded = <<>>
                       ELSE forwarded = seen
===============================================================================
